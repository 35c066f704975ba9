"""Benchmark configurations and seeded synthetic inputs.

The five configurations are the reference path's headline shapes (the
reference's own benchmark is benchmark/bench_attention.py of
JoursBleu/rocm_attn; its README quotes B=1,H=32,L=2048,D=128 fp16,
README.md:51-73).  Inputs are synthetic: i.i.d. normal values drawn slice by
slice, one CPU ``torch.Generator`` per (tensor, batch, head) seeded by a fixed
function of (seed, tensor, b, h).  Any process can therefore regenerate any
(b, h) slice on its own -- a rank generates only the heads it owns, and a
checker regenerates exactly the heads it verifies.
"""
from __future__ import annotations

import dataclasses
from typing import Iterable, Optional, Sequence

import torch

DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}


@dataclasses.dataclass(frozen=True)
class Shape:
    B: int
    H: int
    Lq: int
    Lk: int
    D: int

    @property
    def bh(self) -> int:
        return self.B * self.H

    def flops(self, causal: bool) -> float:
        """Algorithmic FLOPs: 4*D per unmasked score (2*D for QK^T, 2*D for PV).
        Causal counts exactly the unmasked (i, j <= i) pairs."""
        return 4.0 * self.D * self.bh * self.unmasked_pairs(causal)

    def unmasked_pairs(self, causal: bool) -> float:
        if not causal:
            return float(self.Lq) * self.Lk
        # rows i < Lk see i+1 keys, rows i >= Lk see all Lk keys
        n = min(self.Lq, self.Lk)
        return n * (n + 1) / 2.0 + max(0, self.Lq - self.Lk) * float(self.Lk)

    def io_bytes(self, elem: int = 2) -> float:
        """Algorithmic HBM bytes: read Q, K, V once and write O once."""
        return float(elem) * self.bh * self.D * (2 * self.Lq + 2 * self.Lk)


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    shapes: tuple
    dtype: str
    causal: bool
    value_scale: float = 1.0  # inputs are N(0,1) * value_scale

    def flops(self) -> float:
        return sum(s.flops(self.causal) for s in self.shapes)


WORKLOADS = {
    "c1": Workload("c1-noncausal-B1-H32-L2048-D128-fp16", (Shape(1, 32, 2048, 2048, 128),), "fp16", False),
    "c2": Workload("c2-causal-B1-H32-L2048-D128-fp16", (Shape(1, 32, 2048, 2048, 128),), "fp16", True),
    "c3": Workload("c3-noncausal-B8-H16-L1024-D64-bf16", (Shape(8, 16, 1024, 1024, 64),), "bf16", False, 0.5),
    "c4": Workload("c4-causal-B1-H64-L16384-D128-fp16", (Shape(1, 64, 16384, 16384, 128),), "fp16", True),
    "c5": Workload("c5-sweep-noncausal-fp16",
                   (Shape(2, 16, 256, 256, 64), Shape(4, 16, 512, 512, 64), Shape(1, 32, 4096, 4096, 128),
                    Shape(16, 8, 128, 128, 128), Shape(1, 32, 8192, 8192, 128)), "fp16", False),
}

# The reference's inference shape set for its production caller, UnifoLM-WMA
# (benchmark/attn_shapes_unifolm_infer.txt:1-17, run by
# benchmark/run_preset_benchmarks.sh:7-22 as fp16, non-causal): huge B*H with
# short sequences, and cross attention with 93 or 351 keys.
UNIFOLM_SHAPES = (
    "2560,8,16,64;16,5,2560,64;2560,5,16,64;16,10,640,64;640,10,16,64;16,20,160,64;160,20,16,64;"
    "16,20,40,64;40,20,16,64;16,5,2560,93,64;16,10,640,93,64;16,20,160,93,64;16,20,40,93,64;"
    "16,5,2560,351,64;16,10,640,351,64;16,20,160,351,64;16,20,40,351,64"
)

_TENSOR_ID = {"q": 0, "k": 1, "v": 2}


def slice_seed(seed: int, tensor: str, b: int, h: int) -> int:
    """Seed of the (tensor, b, h) slice; distinct for distinct arguments."""
    return (((seed * 3 + _TENSOR_ID[tensor]) * 1_000_003 + b) * 100_003 + h) % (2 ** 63 - 1)


def make_slice(seed: int, tensor: str, b: int, h: int, L: int, D: int, dtype: torch.dtype,
               value_scale: float = 1.0) -> torch.Tensor:
    g = torch.Generator(device="cpu")
    g.manual_seed(slice_seed(seed, tensor, b, h))
    x = torch.randn(L, D, generator=g, dtype=torch.float32)
    if value_scale != 1.0:
        x = x * value_scale
    return x.to(dtype)


def make_qkv(shape: Shape, dtype: torch.dtype, seed: int = 0, value_scale: float = 1.0,
             bh_range: Optional[Sequence[int]] = None, device: str | torch.device = "cpu"):
    """q [B', 1, Lq, D] ... for the flattened (b*H + h) indices in ``bh_range``
    (all of them by default), stacked as [1, len(bh_range), L, D] when a range
    is given and [B, H, L, D] otherwise."""
    idx = list(range(shape.bh)) if bh_range is None else list(bh_range)
    out = []
    for name, L in (("q", shape.Lq), ("k", shape.Lk), ("v", shape.Lk)):
        t = torch.empty(len(idx), L, shape.D, dtype=dtype, device=device)
        for i, f in enumerate(idx):
            t[i].copy_(make_slice(seed, name, f // shape.H, f % shape.H, L, shape.D, dtype, value_scale))
        if bh_range is None:
            t = t.view(shape.B, shape.H, L, shape.D)
        else:
            t = t.view(1, len(idx), L, shape.D)
        out.append(t)
    return tuple(out)


def shard_range(n_units: int, world: int, rank: int) -> range:
    """Contiguous block partition of ``n_units`` (batch*head) slices over
    ``world`` ranks; sizes differ by at most one and concatenate in order."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    lo = n_units * rank // world
    hi = n_units * (rank + 1) // world
    return range(lo, hi)


def parse_shapes(spec: str) -> list[Shape]:
    """``B,H,Lq,D`` or ``B,H,Lq,Lk,D`` entries separated by ';' -- the
    reference benchmark's --shapes syntax (benchmark/bench_attention.py:25-44)."""
    shapes = []
    for part in spec.split(";"):
        part = part.strip()
        if not part:
            continue
        vals = [int(x) for x in part.split(",")]
        if len(vals) == 4:
            b, h, lq, d = vals
            lk = lq
        elif len(vals) == 5:
            b, h, lq, lk, d = vals
        else:
            raise ValueError("Invalid --shapes entry. Expected B,H,Lq,D or B,H,Lq,Lk,D; got: " + part)
        shapes.append(Shape(b, h, lq, lk, d))
    if not shapes:
        raise ValueError("--shapes is empty")
    return shapes


WORKLOADS["unifolm"] = Workload("unifolm-infer-17-shapes-noncausal-fp16", tuple(parse_shapes(UNIFOLM_SHAPES)),
                                "fp16", False)


def iter_flops(shapes: Iterable[Shape], causal: bool) -> float:
    return sum(s.flops(causal) for s in shapes)
