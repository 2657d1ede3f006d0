"""CPU stand-in for the device steps of d3moe.ep (test infrastructure only).

It lets the expert-parallel exchange (plan, all_to_all_v dispatch, expert
compute on the owner, return, combine) run on gloo CPU ranks. The arithmetic
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
    def router_logits(self, x, router_weight):
        return _bf16(O.router_logits(_np(x), _np(router_weight)))

    def route(self, logits, k, bias=None):
        w, ids = O.route(_np(logits), k, None if bias is None else bias.numpy())
        return _bf16(O.bf16_round(w)), torch.from_numpy(ids)

    def plan(self, ids, experts_per_rank, ranks):
        flat = ids.reshape(-1).numpy()
        dest = flat // experts_per_rank
        order = np.argsort(dest, kind="stable").astype(np.int32)
        counts = np.bincount(dest, minlength=ranks).astype(np.int32)
        inv = np.empty_like(order)
        inv[order] = np.arange(order.size, dtype=np.int32)
        local = (flat[order] % experts_per_rank).astype(np.int64)
        return (torch.from_numpy(counts), torch.from_numpy(order), torch.from_numpy(inv),
                torch.from_numpy(local))

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

    def pack(self, x, ids, weights, experts_per_rank, ranks):
        """The packed dispatch rows of d3_ep_pack, built from dispatch_meta."""
        from d3moe.ep import ep_row_bytes
        T, H = x.shape
        k = ids.shape[1]
        rb = ep_row_bytes(H, k)
        meta_ids, meta_w = self.dispatch_meta(ids, weights, experts_per_rank, ranks)
        send = torch.zeros((ranks, T, rb), dtype=torch.uint8)
        xb = x.contiguous().view(torch.uint8).reshape(T, 2 * H)
        for d in range(ranks):
            send[d, :, : 2 * H] = xb
            send[d, :, 2 * H: 2 * H + 8 * k] = meta_ids[d].contiguous().view(torch.uint8).reshape(T, 8 * k)
            send[d, :, 2 * H + 8 * k: 2 * H + 10 * k] = meta_w[d].contiguous().view(torch.uint8).reshape(T, 2 * k)
        return send.reshape(ranks, T * rb)

    def unpack(self, recv, rows, k, H):
        from d3moe.ep import ep_row_bytes
        rb = ep_row_bytes(H, k)
        r = recv.reshape(rows, rb)
        x = r[:, : 2 * H].contiguous().view(torch.bfloat16)
        ids = r[:, 2 * H: 2 * H + 8 * k].contiguous().view(torch.int64)
        w = r[:, 2 * H + 8 * k: 2 * H + 10 * k].contiguous().view(torch.bfloat16)
        return x, ids, w

    def local_experts_k(self, rows, ids, weights, experts):
        """Oracle expert sum over each row's valid ids (-1 = not routed here)."""
        r = _np(rows)
        idn = ids.numpy()
        w = _np(weights)
        M, k = idn.shape
        ex = experts.ex
        q, sx = O.quant_act_fp8(r)
        acc = np.zeros_like(r)
        for j in range(k):
            valid = idn[:, j] >= 0
            if not valid.any():
                continue
            sel = np.nonzero(valid)[0]
            e_ids = idn[sel, j].reshape(-1, 1)
            gu = O.expert_gate_up(q[sel], sx[sel], ex.w13, ex.s13, e_ids)
            a, sa = O.silu_mul_quant(gu)
            d = O.expert_down_rows(a, sa, ex.w2, ex.s2, e_ids)
            acc[sel] = (acc[sel] + d * w[sel, j: j + 1]).astype(np.float32)
        return _bf16(O.bf16_round(acc))

    def gather_rows(self, x, sorted_pairs, k):
        return x[sorted_pairs.long() // k].clone()

    def local_experts(self, rows, local_ids, experts):
        M = rows.shape[0]
        out, _ = O.moe_experts(_np(rows), local_ids.numpy().reshape(M, 1), np.ones((M, 1), np.float32),
                               experts.ex)
        return _bf16(out)

    def shared_expert(self, x, shared):
        T = x.shape[0]
        out, _ = O.moe_experts(_np(x), np.zeros((T, 1), np.int64), np.ones((T, 1), np.float32), shared.ex)
        return _bf16(out)

    def combine(self, rows, inv, weights, shared, gate):
        T, k = weights.shape
        r = _np(rows)
        w = _np(weights)
        acc = np.zeros((T, r.shape[1]), np.float32)
        invn = inv.numpy()
        for j in range(k):
            acc = (acc + r[invn[np.arange(T) * k + j]] * w[:, j: j + 1]).astype(np.float32)
        routed = O.bf16_round(acc)
        return _bf16(O.combine_experts(routed, _np(shared), _np(gate).reshape(-1)))
