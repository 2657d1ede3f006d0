"""Expert-parallel layer on CPU ranks (gloo, world_size 2 and 4).

The device steps are replaced by the oracle (tests/ep_cpu_ops.py); what is under
test is d3moe.ep's exchange logic: bucketing pairs by owner rank, the counts
all_to_all, the all_to_all_v dispatch and return, and the rank-order combine.
The EP output must equal the single-process oracle layer in routing (exactly)
and values (within the parity tolerance), and a rank that never joins must
surface as an error on the host, not a hang.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]
E, I, H, K, T = 8, 128, 256, 2, 5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer():
    from oracle import moe_oracle as O
    ex = O.Experts({}, {}, {}, {})
    for e in range(E):
        ex.w13[e], ex.s13[e] = O.synth_expert(31, e, 2 * I, H)
        ex.w2[e], ex.s2[e] = O.synth_expert(32, e, H, I)
    sh = O.Experts({}, {}, {}, {})
    sh.w13[0], sh.s13[0] = O.synth_expert(33, 0, 2 * I, H)
    sh.w2[0], sh.s2[0] = O.synth_expert(34, 0, H, I)
    router = O.bf16_round((O.hash_uniform(35, (E + 1, H)) * 0.2).astype(np.float32))
    return ex, sh, router


def _worker(rank, world, port, result_dir, mode, biased=False):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "drama-3-single-b300-inference_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from ep_cpu_ops import CpuEPOps, CpuExperts, _bf16
    from oracle import moe_oracle as O
    from d3moe.ep import ExpertParallelMoE

    ex, sh, router = _layer()
    n = E // world
    local = O.Experts({i: ex.w13[rank * n + i] for i in range(n)}, {i: ex.s13[rank * n + i] for i in range(n)},
                      {i: ex.w2[rank * n + i] for i in range(n)}, {i: ex.s2[rank * n + i] for i in range(n)})
    rng = np.random.default_rng(100 + rank)
    rows = T + rank if mode == "exact" else T  # ragged token counts where the mode allows them
    x = O.bf16_round(rng.standard_normal((rows, H)).astype(np.float32))
    # per-expert router bias, N(0,1) like the 24-layer benchmark stack's
    bias = np.random.default_rng(7).standard_normal(E).astype(np.float32) if biased else None
    layer = ExpertParallelMoE(_bf16(router), CpuExperts(local, n, I, H), CpuExperts(sh, 1, I, H), E, K,
                              ops=CpuEPOps(), mode=mode,
                              router_bias=None if bias is None else torch.from_numpy(bias))
    out, ids, w = layer.forward(_bf16(x), return_routing=True)
    ref, ids_ref, w_ref = O.moe_layer(x, router, ex, sh, K, bias=bias)
    np.save(Path(result_dir) / f"r{rank}.npy", np.stack([out.float().numpy(), ref]))
    np.save(Path(result_dir) / f"ids{rank}.npy", np.stack([ids.numpy(), ids_ref]))
    np.save(Path(result_dir) / f"w{rank}.npy", np.stack([w.float().numpy(), w_ref]))
    dist.barrier()
    dist.destroy_process_group()


def _check_ranks(tmp_path, world):
    for r in range(world):
        out, ref = np.load(tmp_path / f"r{r}.npy")
        ids, ids_ref = np.load(tmp_path / f"ids{r}.npy")
        np.testing.assert_array_equal(ids, ids_ref)
        w, w_ref = np.load(tmp_path / f"w{r}.npy")  # bf16 routing weights, bit-exact
        np.testing.assert_array_equal(w, w_ref)
        err = np.abs(out - ref).max()
        rel = np.sqrt(((out - ref) ** 2).sum() / (ref ** 2).sum())
        assert err <= 2e-2 and rel <= 1e-2, (r, err, rel)


@pytest.mark.parametrize("mode", ["capacity", "exact"])
@pytest.mark.parametrize("world", [2, 4])
def test_ep_layer_matches_single_process_oracle(tmp_path, world, mode):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), mode), nprocs=world, join=True)
    _check_ranks(tmp_path, world)


@pytest.mark.parametrize("mode", ["capacity", "exact"])
def test_ep_layer_with_router_bias_matches_oracle(tmp_path, mode):
    """The router bias enters before the bf16 rounding of the logits on every
    rank, as in the single-GPU layer, so routing stays exact."""
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), mode, True), nprocs=2, join=True)
    _check_ranks(tmp_path, 2)


def _lonely_worker(rank, world, port, result_dir):
    """Both ranks finish one step (a barrier), then rank 1 leaves; rank 0's
    next layer call must end with an error from its process-group timeout
    instead of hanging."""
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "drama-3-single-b300-inference_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    outcome = "no error"
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        dist.barrier()
        if rank == 1:
            return  # leaves between steps, before any collective of the layer
        from ep_cpu_ops import CpuEPOps, CpuExperts, _bf16
        from oracle import moe_oracle as O
        from d3moe.ep import ExpertParallelMoE

        ex, sh, router = _layer()
        n = E // world
        local = O.Experts({i: ex.w13[i] for i in range(n)}, {i: ex.s13[i] for i in range(n)},
                          {i: ex.w2[i] for i in range(n)}, {i: ex.s2[i] for i in range(n)})
        layer = ExpertParallelMoE(_bf16(router), CpuExperts(local, n, I, H), CpuExperts(sh, 1, I, H), E, K,
                                  ops=CpuEPOps(), mode="exact")
        x = O.bf16_round(np.ones((T, H), np.float32))
        layer.forward(_bf16(x))
    except Exception as exc:  # noqa: BLE001 - the error type is the backend's
        outcome = f"error: {type(exc).__name__}"
    if rank == 0:
        (Path(result_dir) / "outcome.txt").write_text(outcome)


def test_ep_missing_rank_fails_with_timeout_not_hang(tmp_path):
    """Rank 0 must not hang: it either raises (written to outcome.txt) or is
    ended by the collective backend (gloo may abort the process when its peer
    is gone); both happen well inside the bound below."""
    ctx = mp.spawn(_lonely_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False)
    ended_by_backend = False
    deadline = 120.0
    import time

    t0 = time.monotonic()
    while time.monotonic() - t0 < deadline:
        try:
            if ctx.join(timeout=5):
                break
        except mp.ProcessExitedException:
            ended_by_backend = True
            break
    hung = [p for p in ctx.processes if p.is_alive()]
    for p in hung:
        p.kill()
    assert not hung, "a rank was still waiting after the deadline"
    out = tmp_path / "outcome.txt"
    if out.exists():
        assert out.read_text().startswith("error"), out.read_text()
    else:
        assert ended_by_backend
