"""Expert-parallel (EP) MoE layer over torch.distributed (NCCL on NVLink).

The reference runs the whole MoE on one GPU. Here the 128 routed experts are
sharded contiguously over the N ranks of a process group (rank r owns experts
[r*E/N, (r+1)*E/N)); the router, the shared expert and the dense projections
are replicated. One layer call on rank r, for its own T tokens:

  1. logits = router(x) bf16 [T, E+1]; top-k routing on the first E columns
     (identical arithmetic on every rank, so routing matches the 1-GPU layer
     bit for bit);
  2. dispatch: each token is quantised once (1x128 E4M3 groups with fp32
     scales, the bytes the expert pipeline would produce itself) and one
     packed row per destination rank carries those bytes, the scales and the
     token's routing restricted to that rank (owner-local ids or -1, the
     routing weight or 0): 2192 bytes a row at H=2048, k=8
     (d3_ep_pack_fp8); one all_to_all moves the rows;
  3. the owner runs its experts straight on the received bytes
     (d3_ep_unpack_fp8, d3_moe_experts_fp8) and produces one weighted partial
     row per received row, bf16(sum over its experts of w * down);
  4. the partials go back with the mirror all_to_all;
  5. d3_combine_pairs on the token's own rank: bf16(sum of its partials in
     rank order) + the gated shared expert, which ran on a side stream while
     the exchange was in flight.

Two ways to choose the destination rows:

  mode="capacity" (default, decode): every token goes to every rank (fixed
  buffers, [N, T] rows), so there is no host synchronisation and the layer,
  NCCL calls included, can be captured into a CUDA graph. All ranks must call
  it with the same T.

  mode="exact" (prefill): a token goes only to the ranks that own at least
  one of its experts (d3_ep_plan_rows: rows ordered by destination rank, a
  slot map per (token, rank)); the row counts are exchanged first and read on
  the host (one synchronisation per call), then the rows move with
  all_to_all_v. Ranks may hold different T.

`ops` is injectable so the exchange logic can be exercised with CPU ranks
(gloo) in tests; the default runs on the GPU.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops as _ops
from ._lib import call


def ep_row_bytes_fp8(H: int, k: int) -> int:
    """Bytes per FP8 packed dispatch row: e4m3 x (H) + H/128 f32 group scales
    + k int64 ids + k bf16 weights, rounded up to 16 (d3_ep_row_bytes_fp8)."""
    return (H + 4 * (H // 128) + 10 * k + 15) // 16 * 16


class CudaEPOps:
    """Device steps of the EP layer on the current CUDA stream."""

    def router_logits(self, x, router_weight, bias=None):
        """bf16 logits [T, E+1]; bias f32 [E] enters before the bf16 rounding."""
        return _ops.router_logits(x, router_weight, bias)

    def route(self, logits, k, bias=None):
        return _ops.route_topk(logits, k, bias=bias, weights_dtype=torch.bfloat16)

    def plan_rows(self, ids, experts_per_rank, ranks):
        """(send_counts int32 [ranks], slot int32 [T, ranks]) of d3_ep_plan_rows."""
        T, k = ids.shape
        dev = ids.device
        send_counts = torch.empty(ranks, dtype=torch.int32, device=dev)
        slot = torch.empty((T, ranks), dtype=torch.int32, device=dev)
        call("d3_ep_plan_rows", ids.data_ptr(), T, k, experts_per_rank, ranks, send_counts.data_ptr(),
             slot.data_ptr(), _ops._stream(dev))
        return send_counts, slot

    def pack_fp8(self, x, ids, weights, experts_per_rank, ranks, slot=None, rows=None):
        """FP8 packed send rows, uint8 [ranks, T * row_bytes] (every token to
        every rank), or [rows, row_bytes] placed by a plan_rows slot map."""
        T, H = x.shape
        k = ids.shape[1]
        rb = ep_row_bytes_fp8(H, k)
        shape = (ranks, T * rb) if slot is None else (rows, rb)
        send = torch.empty(shape, dtype=torch.uint8, device=x.device)
        call("d3_ep_pack_fp8", x.data_ptr(), _ops._row_stride(x), ids.data_ptr(),
             weights.contiguous().data_ptr(), T, k, H, experts_per_rank, ranks,
             None if slot is None else slot.data_ptr(), send.data_ptr(), _ops._stream(x.device))
        return send

    def unpack_fp8(self, recv, rows, k, H):
        """Received FP8 rows -> (q e4m3 [rows, H] strided view, scales f32
        [rows, H/128], ids int64 [rows, k], weights bf16 [rows, k])."""
        rb = ep_row_bytes_fp8(H, k)
        scales = torch.empty((rows, H // 128), dtype=torch.float32, device=recv.device)
        ids = torch.empty((rows, k), dtype=torch.int64, device=recv.device)
        w = torch.empty((rows, k), dtype=torch.bfloat16, device=recv.device)
        call("d3_ep_unpack_fp8", recv.data_ptr(), rows, k, H, scales.data_ptr(), ids.data_ptr(),
             w.data_ptr(), _ops._stream(recv.device))
        q = recv.view(rows, rb)[:, :H].view(torch.float8_e4m3fn)
        return q, scales, ids, w

    def local_experts_fp8(self, q, scales, ids, weights, experts):
        """Weighted sum over each received row's local experts (ids -1
        skipped), on the received E4M3 bytes."""
        return _ops.moe_experts_fp8(q, scales, ids, weights, experts, transposed=False)

    def dispatch_meta(self, ids, weights, experts_per_rank, ranks):
        T, k = ids.shape
        meta_ids = torch.empty((ranks, T, k), dtype=torch.int64, device=ids.device)
        meta_w = torch.empty((ranks, T, k), dtype=torch.bfloat16, device=ids.device)
        call("d3_ep_dispatch_meta", ids.data_ptr(), weights.contiguous().data_ptr(), T, k, experts_per_rank,
             ranks, meta_ids.data_ptr(), meta_w.data_ptr(), _ops._stream(ids.device))
        return meta_ids, meta_w

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
    ...). shared: the shared expert (E = 1), replicated. router_bias:
    optional per-expert f32 [E], added to the router logits before their bf16
    rounding (as d3_moe_layer does), so routing matches the 1-GPU layer."""

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
        # f32 [E], added to the router logits before their bf16 rounding, as
        # in the single-GPU layer
        self.router_bias = None if router_bias is None else router_bias.to(torch.float32).contiguous()
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
        logits = ops.router_logits(x, self.router, self.router_bias)
        weights, ids = ops.route(logits[:, : self.E], self.k)
        shared, side = self._shared_begin(x)
        send = ops.pack_fp8(x, ids, weights, self.E_local, N)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        q, qs, ids_recv, w_recv = ops.unpack_fp8(recv, N * T, self.k, H)
        partial = ops.local_experts_fp8(q, qs, ids_recv, w_recv, self.experts)
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
        N = self.world
        T, H = x.shape
        logits = ops.router_logits(x, self.router, self.router_bias)
        weights, ids = ops.route(logits[:, : self.E], self.k)
        send_counts_dev, slot = ops.plan_rows(ids, self.E_local, N)
        shared, side = self._shared_begin(x)
        # row counts: device -> all_to_all -> host (the one host synchronisation)
        counts64 = send_counts_dev.to(torch.int64)
        recv_counts_dev = torch.empty_like(counts64)
        dist.all_to_all_single(recv_counts_dev, counts64, group=self.group)
        both = torch.stack([counts64, recv_counts_dev]).cpu()
        send_counts = [int(v) for v in both[0]]
        recv_counts = [int(v) for v in both[1]]
        send = ops.pack_fp8(x, ids, weights, self.E_local, N, slot=slot, rows=sum(send_counts))
        recv = self._exchange(send, send_counts, recv_counts)
        R = recv.shape[0]
        if R:
            q, qs, ids_recv, w_recv = ops.unpack_fp8(recv, R, self.k, H)
            partial = ops.local_experts_fp8(q, qs, ids_recv, w_recv, self.experts)
        else:
            partial = torch.empty((0, H), dtype=torch.bfloat16, device=x.device)
        rows_back = self._exchange(partial, recv_counts, send_counts)
        shared = self._shared_end(shared, side)
        ones = self._combine_inputs(T, x.device)[1]
        out = ops.combine(rows_back, slot.reshape(-1), ones, shared, logits[:, self.E: self.E + 1])
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
