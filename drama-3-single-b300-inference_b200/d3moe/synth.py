"""Seeded synthetic weights for one FP8 MoE layer (the shapes and value
distributions of the benchmark configurations): N(0, 0.02) matrices quantised
into e4m3 with fp32 128x128 block scales (scale = amax / 448), bf16 router.

Generation runs on the target device with a seeded torch.Generator, so a
layer of 128 experts (~600 MB of FP8) is made in well under a second.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

FP8 = torch.float8_e4m3fn


@dataclass
class ExpertWeights:
    """The reference's expert container (src/drama3/kernels.py:336-350)."""

    w13_weight: torch.Tensor     # [E, 2I, H] e4m3, rows [gate | up]
    w13_scale_inv: torch.Tensor  # [E, 2I/128, H/128] f32
    w2_weight: torch.Tensor      # [E, H, I] e4m3
    w2_scale_inv: torch.Tensor   # [E, H/128, I/128] f32

    @property
    def num_experts(self) -> int:
        return self.w13_weight.shape[0]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in
                   (self.w13_weight, self.w13_scale_inv, self.w2_weight, self.w2_scale_inv))


def block_quantize(w: torch.Tensor):
    """fp32 [..., R, C] -> (e4m3 [..., R, C], f32 [..., R/128, C/128]) with
    scale = max(amax, 1e-8)/448 per 128x128 block (experimental_fp8.py:15-18)."""
    *lead, R, C = w.shape
    b = w.reshape(*lead, R // 128, 128, C // 128, 128)
    amax = b.abs().amax(dim=(-3, -1))
    scale = torch.clamp(amax, min=1e-8) / 448.0
    q = (b / scale[..., :, None, :, None]).clamp(-448.0, 448.0).to(FP8)
    return q.reshape(*lead, R, C), scale.to(torch.float32).contiguous()


def make_experts(E: int, I: int, H: int, seed: int, device, std: float = 0.02,
                 chunk: int = 16) -> ExpertWeights:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    w13 = torch.empty((E, 2 * I, H), dtype=FP8, device=device)
    s13 = torch.empty((E, 2 * I // 128, H // 128), dtype=torch.float32, device=device)
    w2 = torch.empty((E, H, I), dtype=FP8, device=device)
    s2 = torch.empty((E, H // 128, I // 128), dtype=torch.float32, device=device)
    for e0 in range(0, E, chunk):
        e1 = min(E, e0 + chunk)
        a = torch.randn((e1 - e0, 2 * I, H), generator=gen, device=device) * std
        w13[e0:e1], s13[e0:e1] = block_quantize(a)
        b = torch.randn((e1 - e0, H, I), generator=gen, device=device) * std
        w2[e0:e1], s2[e0:e1] = block_quantize(b)
        del a, b
    return ExpertWeights(w13, s13, w2, s2)


@dataclass
class LayerWeights:
    """One MoE layer: routed experts, the shared expert (E = 1) and the packed
    bf16 router projection [E+1, H] (rows 0..E-1 router, row E the shared
    expert gate, like the packed projection of src/drama3/model.py:236-245)."""

    experts: ExpertWeights
    shared: ExpertWeights
    router: torch.Tensor
    router_bias: torch.Tensor | None = None

    def nbytes(self) -> int:
        n = self.experts.nbytes() + self.shared.nbytes() + self.router.numel() * 2
        return n + (0 if self.router_bias is None else self.router_bias.numel() * 4)


def make_layer(E: int = 128, I: int = 768, H: int = 2048, seed: int = 0, device="cuda",
               router_bias: str | None = None) -> LayerWeights:
    """Synthetic layer. router_bias: None, "normal" (per-expert N(0,1)) or
    "zipf" (log of a Zipf(s=1.1) distribution over a random expert order)."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    router = (torch.randn((E + 1, H), generator=gen) * 0.02).to(torch.bfloat16).to(device)
    bias = None
    if router_bias == "normal":
        bias = torch.randn(E, generator=gen).to(device)
    elif router_bias == "zipf":
        perm = torch.randperm(E, generator=gen)
        ranks = torch.empty(E)
        ranks[perm] = torch.arange(1, E + 1, dtype=torch.float32)
        p = ranks.pow(-1.1)
        bias = torch.log(p / p.sum()).to(device)
    experts = make_experts(E, I, H, seed * 1000 + 1, device)
    shared = make_experts(1, I, H, seed * 1000 + 2, device)
    return LayerWeights(experts, shared, router.contiguous(), bias)
