"""Expert-parallel layer on GPUs (NCCL): its output must match the single-GPU
fused layer on the same tokens (routing exactly, values within tolerance).
The one-rank case runs on any box with a GPU; the multi-rank case needs at
least two GPUs and is skipped otherwise."""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
E, I, H, K = 128, 768, 2048, 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir, T, mode="capacity"):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "drama-3-single-b300-inference_b200")]
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    from d3moe import ops, synth
    from d3moe.ep import ExpertParallelMoE, shard_experts

    lw = synth.make_layer(E, I, H, seed=5, device=dev)
    layer = ExpertParallelMoE(lw.router, shard_experts(lw.experts, rank, world), lw.shared, E, K, mode=mode)
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    rows = T + 3 * rank if mode == "exact" else T
    x = torch.randn((rows, H), generator=g, device=dev).to(torch.bfloat16)
    out, ids, w = layer.forward(x, return_routing=True)
    ref, ids_ref, w_ref = ops.moe_layer(x, lw.router, lw.experts, lw.shared, K, return_routing=True)
    torch.cuda.synchronize()
    np.save(Path(result_dir) / f"r{rank}.npy", np.stack([out.float().cpu().numpy(), ref.float().cpu().numpy()]))
    np.save(Path(result_dir) / f"ids{rank}.npy", np.stack([ids.cpu().numpy(), ids_ref.cpu().numpy()]))
    dist.barrier()
    dist.destroy_process_group()


def _check(result_dir, world):
    for r in range(world):
        out, ref = np.load(Path(result_dir) / f"r{r}.npy")
        ids, ids_ref = np.load(Path(result_dir) / f"ids{r}.npy")
        np.testing.assert_array_equal(ids, ids_ref)
        err = np.abs(out - ref).max()
        rel = np.sqrt(((out - ref) ** 2).sum() / (ref ** 2).sum())
        assert err <= 2e-2 and rel <= 1e-2, (r, err, rel)


@pytest.mark.parametrize("mode", ["capacity", "exact"])
def test_ep_one_rank_matches_fused_layer(tmp_path, mode):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(1, _free_port(), str(tmp_path), 64, mode), nprocs=1, join=True)
    _check(tmp_path, 1)


@pytest.mark.parametrize("mode", ["capacity", "exact"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_multi_rank_matches_fused_layer(tmp_path, world, mode):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), 64, mode), nprocs=world, join=True)
    _check(tmp_path, world)


def test_ep_pack_unpack_matches_dispatch_meta():
    """The packed dispatch rows carry exactly dispatch_meta's per-rank routing
    and the token rows (d3_ep_pack / d3_ep_unpack_meta round trip)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe.ep import CudaEPOps
    ops = CudaEPOps()
    T, H, k, N, epr = 37, 2048, 8, 4, 32
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    x = torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)
    ids = torch.randint(0, N * epr, (T, k), generator=g, device="cuda")
    ids[3, 2] = -1  # an empty slot
    w = torch.rand((T, k), generator=g, device="cuda").to(torch.bfloat16)
    send = ops.pack(x, ids, w, epr, N)
    rows, ids_u, w_u = ops.unpack(send, N * T, k, H)
    meta_ids, meta_w = ops.dispatch_meta(ids, w, epr, N)
    torch.cuda.synchronize()
    assert torch.equal(ids_u, meta_ids.view(N * T, k))
    assert torch.equal(w_u, meta_w.view(N * T, k))
    assert torch.equal(rows, x.unsqueeze(0).expand(N, T, H).reshape(N * T, H))
