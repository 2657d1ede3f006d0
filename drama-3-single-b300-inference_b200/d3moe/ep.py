"""Expert-parallel (EP) MoE layer over torch.distributed (NCCL on NVLink).

The reference runs the whole MoE on one GPU. Here the 128 routed experts are
sharded contiguously over the N ranks of a process group (rank r owns experts
[r*E/N, (r+1)*E/N)); the router, the shared expert and the dense projections
are replicated. One layer call on rank r, for its own T tokens:

  1. logits = router(x) bf16 [T, E+1]; top-k routing on the first E columns
     (identical arithmetic on every rank, so routing matches the 1-GPU layer
     bit for bit);
  2. ep_plan buckets the T*k (token, expert) pairs by owner rank, stable;
  3. send counts are exchanged (all_to_all, one small host read), then the
     bf16 token rows and the owner-local expert ids (all_to_all_v);
  4. the owner runs its experts on the rows it received (top-1 per row, weight
     1, so each row comes back as bf16(down(...)) of one (token, expert) pair);
  5. the rows go back with the mirror all_to_all_v;
  6. combine_pairs: bf16(sum_r w[t,r] * row) in rank order + gated shared
     expert, on the token's own rank.

That is mode="exact": it moves only the pairs, but needs a host read of the
send counts per call. The default, mode="capacity", has no host
synchronisation (so the layer can be captured into a CUDA graph with its NCCL
calls): every token row goes once to every rank together with the routing
restricted to that rank's experts (local ids or -1, the routing weight or 0),
packed with the row into one buffer so the dispatch is a single all_to_all
(d3_ep_pack / d3_ep_unpack_meta); the owner runs its experts on all received
rows with those k ids and returns one weighted partial row per token,
bf16(sum over its experts of w * down), and the token's rank adds the N
partials in rank order plus the gated shared expert (d3_combine_pairs with
weight 1 per rank). The shared expert runs on a side stream while the
exchange is in flight. All ranks must call the layer with the same T. At
decode sizes this moves T*N rows per rank per direction, the same order as the
exact scheme.

The device steps are the C ABI entry points d3_ep_plan, d3_ep_pack,
d3_ep_unpack_meta, d3_ep_dispatch_meta, d3_gather_rows, d3_moe_experts and
d3_combine_pairs. `ops` is injectable so the
exchange logic can be exercised with CPU ranks (gloo) in tests; the default
runs on the GPU.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops as _ops
from ._lib import call


def ep_row_bytes(H: int, k: int) -> int:
    """Bytes per packed dispatch row: x (2H) + k int64 ids + k bf16 weights,
    rounded up to 16 (d3_ep_row_bytes)."""
    return (2 * H + 10 * k + 15) // 16 * 16


class CudaEPOps:
    """Device steps of the EP layer on the current CUDA stream."""

    def router_logits(self, x, router_weight):
        return _ops.router_logits(x, router_weight)

    def route(self, logits, k, bias=None):
        return _ops.route_topk(logits, k, bias=bias, weights_dtype=torch.bfloat16)

    def plan(self, ids, experts_per_rank, ranks):
        T, k = ids.shape
        P = T * k
        dev = ids.device
        i32 = dict(dtype=torch.int32, device=dev)
        send_counts = torch.empty(ranks, **i32)
        send_starts = torch.empty(ranks, **i32)
        sorted_pairs = torch.empty(max(P, 1), **i32)
        inv = torch.empty(max(P, 1), **i32)
        local_ids = torch.empty(max(P, 1), dtype=torch.int64, device=dev)
        scratch = torch.empty(P + 1, **i32)
        call("d3_ep_plan", ids.data_ptr(), T, k, experts_per_rank, ranks, send_counts.data_ptr(),
             send_starts.data_ptr(), sorted_pairs.data_ptr(), inv.data_ptr(), local_ids.data_ptr(),
             scratch.data_ptr(), _ops._stream(dev))
        return send_counts, sorted_pairs[:P], inv[:P], local_ids[:P]

    def pack(self, x, ids, weights, experts_per_rank, ranks):
        """Packed capacity-mode send buffer uint8 [ranks, T * row_bytes]."""
        T, H = x.shape
        k = ids.shape[1]
        rb = ep_row_bytes(H, k)
        send = torch.empty((ranks, T * rb), dtype=torch.uint8, device=x.device)
        call("d3_ep_pack", x.data_ptr(), _ops._row_stride(x), ids.data_ptr(),
             weights.contiguous().data_ptr(), T, k, H, experts_per_rank, ranks, send.data_ptr(),
             _ops._stream(x.device))
        return send

    def unpack(self, recv, rows, k, H):
        """Received packed rows -> (x rows bf16 [rows, H] strided view, ids, weights)."""
        rb = ep_row_bytes(H, k)
        ids = torch.empty((rows, k), dtype=torch.int64, device=recv.device)
        w = torch.empty((rows, k), dtype=torch.bfloat16, device=recv.device)
        call("d3_ep_unpack_meta", recv.data_ptr(), rows, k, H, ids.data_ptr(), w.data_ptr(),
             _ops._stream(recv.device))
        return recv.view(rows, rb).view(torch.bfloat16)[:, :H], ids, w

    def gather_rows(self, x, sorted_pairs, k):
        T, H = x.shape
        rows = sorted_pairs.numel()
        out = torch.empty((rows, H), dtype=x.dtype, device=x.device)
        call("d3_gather_rows", x.data_ptr(), x.stride(0), T, H, k, sorted_pairs.data_ptr(), rows,
             out.data_ptr(), _ops._stream(x.device))
        return out

    def dispatch_meta(self, ids, weights, experts_per_rank, ranks):
        T, k = ids.shape
        meta_ids = torch.empty((ranks, T, k), dtype=torch.int64, device=ids.device)
        meta_w = torch.empty((ranks, T, k), dtype=torch.bfloat16, device=ids.device)
        call("d3_ep_dispatch_meta", ids.data_ptr(), weights.contiguous().data_ptr(), T, k, experts_per_rank,
             ranks, meta_ids.data_ptr(), meta_w.data_ptr(), _ops._stream(ids.device))
        return meta_ids, meta_w

    def local_experts_k(self, rows, ids, weights, experts):
        """Weighted sum over each row's (up to k) local experts; ids -1 skipped."""
        out, _ = _ops.moe_experts(rows, ids, weights, experts)
        return out

    def local_experts(self, rows, local_ids, experts):
        M = rows.shape[0]
        ones = torch.ones((M, 1), dtype=torch.bfloat16, device=rows.device)
        out, _ = _ops.moe_experts(rows, local_ids.view(M, 1), ones, experts)
        return out

    def shared_expert(self, x, shared):
        T = x.shape[0]
        zeros = torch.zeros((T, 1), dtype=torch.int64, device=x.device)
        ones = torch.ones((T, 1), dtype=torch.bfloat16, device=x.device)
        out, _ = _ops.moe_experts(x, zeros, ones, shared)
        return out

    def combine(self, rows, inv, weights, shared, gate):
        T, k = weights.shape
        H = rows.shape[1]
        out = torch.empty((T, H), dtype=torch.bfloat16, device=rows.device)
        call("d3_combine_pairs", rows.data_ptr(), inv.data_ptr(), weights.contiguous().data_ptr(), T, k, H,
             None if shared is None else shared.data_ptr(), None if gate is None else gate.data_ptr(),
             0 if gate is None else gate.stride(0), out.data_ptr(), _ops._stream(rows.device))
        return out


class ExpertParallelMoE:
    """One MoE layer with its routed experts sharded over `group`.

    router_weight: bf16 [E+1, H] (router rows + shared-expert gate row),
    replicated. experts_local: this rank's experts (w13_weight [E/N, 2I, H],
    ...). shared: the shared expert (E = 1), replicated."""

    def __init__(self, router_weight, experts_local, shared, num_experts: int, top_k: int = 8,
                 group=None, ops=None, router_bias=None, mode: str = "capacity"):
        if mode not in ("capacity", "exact"):
            raise ValueError("mode must be 'capacity' or 'exact'")
        self.mode = mode
        self._combine_index = {}
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not shard evenly over {self.world} ranks")
        self.E = num_experts
        self.E_local = num_experts // self.world
        if experts_local.w13_weight.shape[0] != self.E_local:
            raise ValueError("experts_local must hold exactly num_experts / world_size experts")
        self.router = router_weight
        self.router_bias = router_bias
        self.experts = experts_local
        self.shared = shared
        self.k = top_k
        self.ops = ops if ops is not None else CudaEPOps()
        self._side = {}

    def _exchange(self, send, send_counts, recv_counts):
        """all_to_all_v of rows (first dim split by counts)."""
        out = send.new_empty((sum(recv_counts),) + tuple(send.shape[1:]))
        dist.all_to_all_single(out, send.contiguous(), recv_counts, send_counts, group=self.group)
        return out

    def forward(self, x, return_routing: bool = False):
        if self.mode == "capacity":
            return self._forward_capacity(x, return_routing)
        return self._forward_exact(x, return_routing)

    def _combine_inputs(self, T, device):
        """Row index (token t, rank d) -> d*T + t and unit weights [T, N]."""
        key = (T, str(device))
        got = self._combine_index.get(key)
        if got is None:
            N = self.world
            t = torch.arange(T, dtype=torch.int32).view(T, 1)
            d = torch.arange(N, dtype=torch.int32).view(1, N)
            inv = (d * T + t).reshape(-1).contiguous().to(device)
            ones = torch.ones((T, N), dtype=torch.bfloat16, device=device)
            got = (inv, ones)
            self._combine_index[key] = got
        return got

    def _shared_begin(self, x):
        """The shared expert on the layer's own rows; on CUDA it runs on a side
        stream so it overlaps the dispatch exchange (joined in _shared_end)."""
        if not x.is_cuda:
            return self.ops.shared_expert(x, self.shared), None
        main = torch.cuda.current_stream(x.device)
        side = self._side.get(x.device)
        if side is None:
            side = torch.cuda.Stream(x.device)
            self._side[x.device] = side
        side.wait_stream(main)
        with torch.cuda.stream(side):
            shared = self.ops.shared_expert(x, self.shared)
        return shared, side

    def _shared_end(self, shared, side):
        if side is not None:
            main = torch.cuda.current_stream(shared.device)
            main.wait_stream(side)
            shared.record_stream(main)
        return shared

    def _forward_capacity(self, x, return_routing: bool):
        ops = self.ops
        N = self.world
        T, H = x.shape
        logits = ops.router_logits(x, self.router)
        weights, ids = ops.route(logits[:, : self.E], self.k, bias=self.router_bias)
        shared, side = self._shared_begin(x)
        if hasattr(ops, "pack"):
            # one exchange of packed rows (token row + per-rank routing)
            send = ops.pack(x, ids, weights, self.E_local, N)
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=self.group)
            rows, ids_recv, w_recv = ops.unpack(recv, N * T, self.k, H)
        else:
            meta_ids, meta_w = ops.dispatch_meta(ids, weights, self.E_local, N)
            x_send = x.unsqueeze(0).expand(N, T, H).contiguous()
            x_recv = torch.empty_like(x_send)
            ids_recv = torch.empty_like(meta_ids)
            w_recv = torch.empty_like(meta_w)
            dist.all_to_all_single(x_recv, x_send, group=self.group)
            dist.all_to_all_single(ids_recv, meta_ids, group=self.group)
            dist.all_to_all_single(w_recv, meta_w, group=self.group)
            rows = x_recv.view(N * T, H)
        partial = ops.local_experts_k(rows, ids_recv.view(N * T, self.k), w_recv.view(N * T, self.k),
                                      self.experts)
        partial_back = torch.empty_like(partial)
        dist.all_to_all_single(partial_back, partial, group=self.group)
        shared = self._shared_end(shared, side)
        inv, ones = self._combine_inputs(T, x.device)
        out = ops.combine(partial_back, inv, ones, shared, logits[:, self.E: self.E + 1])
        if return_routing:
            return out, ids, weights
        return out

    def _forward_exact(self, x, return_routing: bool):
        ops = self.ops
        T, H = x.shape
        logits = ops.router_logits(x, self.router)
        weights, ids = ops.route(logits[:, : self.E], self.k, bias=self.router_bias)
        send_counts_dev, sorted_pairs, inv, local_ids = ops.plan(ids, self.E_local, self.world)
        # counts: device -> all_to_all -> host (the one host synchronisation)
        counts64 = send_counts_dev.to(torch.int64)
        recv_counts_dev = torch.empty_like(counts64)
        dist.all_to_all_single(recv_counts_dev, counts64, group=self.group)
        both = torch.stack([counts64, recv_counts_dev]).cpu()
        send_counts = [int(v) for v in both[0]]
        recv_counts = [int(v) for v in both[1]]
        rows_send = ops.gather_rows(x, sorted_pairs, self.k)
        rows_recv = self._exchange(rows_send, send_counts, recv_counts)
        ids_recv = self._exchange(local_ids, send_counts, recv_counts)
        if rows_recv.shape[0]:
            y_recv = ops.local_experts(rows_recv, ids_recv, self.experts)
        else:
            y_recv = rows_recv
        rows_back = self._exchange(y_recv, recv_counts, send_counts)
        shared = ops.shared_expert(x, self.shared)
        out = ops.combine(rows_back, inv, weights, shared, logits[:, self.E: self.E + 1])
        if return_routing:
            return out, ids, weights
        return out

    __call__ = forward


def shard_experts(experts, rank: int, world: int):
    """The contiguous expert slice rank `rank` owns (views, no copy)."""
    from .synth import ExpertWeights

    E = experts.w13_weight.shape[0]
    n = E // world
    sl = slice(rank * n, (rank + 1) * n)
    return ExpertWeights(experts.w13_weight[sl], experts.w13_scale_inv[sl], experts.w2_weight[sl],
                         experts.w2_scale_inv[sl])
