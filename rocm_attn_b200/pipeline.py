"""Attention on host-resident tensors with the transfers overlapped.

``attn_forward_pinned`` is the public entry for callers whose q/k/v live in
pinned host memory (the end-to-end path of the benchmark).  It splits the
flattened (batch, head) slices into chunks and keeps three CUDA streams busy:
the host-to-device copy of chunk c+1, the attention of chunk c (the caller's
current stream, through ``attn_forward``) and the device-to-host copy of
chunk c-1 run at the same time, so a step costs about the larger of the two
PCIe directions instead of their sum plus the compute.  The reference has no
counterpart: its callers copy whole tensors and call the op
(benchmark/bench_attention.py:178-184).
"""
from __future__ import annotations

import math
import threading
from collections import OrderedDict
from typing import Optional

import torch

_lock = threading.Lock()
_state: "OrderedDict[tuple, dict]" = OrderedDict()
# Device buffer sets kept for reuse (the most recently used ones); a caller
# cycling through more shapes than this reallocates, but memory stays bounded.
MAX_CACHED_SHAPES = 4


def _release(st: dict) -> None:
    """Waits until no queued work can still touch the buffers of an evicted
    entry (its copies and the attention launches that read them), so the
    allocator may hand the memory to someone else."""
    for ev in st["done"].values():
        ev.synchronize()
    st["s_in"].synchronize()
    st["s_out"].synchronize()


def _device_state(device: torch.device, key: tuple, q_shape, k_shape, dtype):
    """Device buffers and events for one (device, shape, dtype, chunking),
    reused across calls so a steady caller allocates nothing."""
    with _lock:
        st = _state.get(key)
        if st is not None:
            _state.move_to_end(key)
        else:
            while len(_state) >= MAX_CACHED_SHAPES:
                _, old = _state.popitem(last=False)
                _release(old)
            st = {
                "q": torch.empty(q_shape, dtype=dtype, device=device),
                "k": torch.empty(k_shape, dtype=dtype, device=device),
                "v": torch.empty(k_shape, dtype=dtype, device=device),
                "s_in": torch.cuda.Stream(device=device),
                "s_out": torch.cuda.Stream(device=device),
                "done": {},  # chunk -> event recorded after its attention was queued
            }
            _state[key] = st
        return st


def _chunk_sizes(BH: int, base: int, uniform: bool) -> list:
    """Slices per chunk.  The step ends with the last chunk's attention and
    device-to-host copy after the last host-to-device copy, so long splits end
    in chunks that halve down to one slice (2*base, base, ..., 1, 1), and the
    bulk before them goes in chunks of 3*base: C4 (64 heads, base 4) runs as
    12,12,12,12,8,4,2,1,1 heads, measured 3 % faster end to end than sixteen
    chunks of 4.  Short splits (fewer than eight chunks), and an explicit
    chunk size, stay uniform."""
    if uniform or BH < 8 * base:
        return [min(base, BH - c0) for c0 in range(0, BH, base)]
    tail = []
    s = 2 * base
    while s >= 1:
        tail.append(s)
        s //= 2
    tail.append(1)
    bulk = BH - sum(tail)
    if bulk <= 0:
        return [min(base, BH - c0) for c0 in range(0, BH, base)]
    big = 3 * base
    return [big] * (bulk // big) + ([bulk % big] if bulk % big else []) + tail


def attn_forward_pinned(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                        scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                        chunk_slices: Optional[int] = None, device: Optional[torch.device] = None) -> torch.Tensor:
    """Attention forward for contiguous pinned host tensors q [B, H, Lq, D],
    k/v [B, H, Lk, D].  Returns O [B, H, Lq, D] in pinned host memory (``out``
    if given).  Asynchronous like the op itself: the result is ready once the
    caller's current stream on ``device`` is synchronised.  ``chunk_slices``
    (batch, head) slices go per chunk (default: a base of one chunk per about
    20 MB of q/k/v, between 2 and 16 chunks, measured best or within 3 % of
    best from 33 MB to 805 MB of inputs, where every chunk adds some host work;
    splits of eight or more chunks end in halving chunks, _chunk_sizes)."""
    from . import attn_forward

    for t in (q, k, v) + ((out,) if out is not None else ()):
        if t.device.type != "cpu" or not t.is_contiguous():
            raise ValueError("attn_forward_pinned takes contiguous host tensors")
        if not t.is_pinned():
            # a pageable buffer turns every chunk copy into a synchronous
            # staged copy, which defeats the overlap this entry point exists for
            raise ValueError("attn_forward_pinned takes pinned host tensors (use .pin_memory())")
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    BH = B * H
    if out is None:
        out = torch.empty((B, H, Lq, D), dtype=q.dtype, pin_memory=True)
    if BH == 0 or Lq == 0:
        return out
    if chunk_slices:
        n = chunk_slices
    else:
        in_bytes = (q.numel() + k.numel() + v.numel()) * q.element_size()
        n_chunks = min(16, max(2, round(in_bytes / 20e6)))
        n = max(1, math.ceil(BH / n_chunks))
    sizes = _chunk_sizes(BH, n, uniform=bool(chunk_slices))
    chunks, c0 = [], 0
    for sz in sizes:
        chunks.append((c0, c0 + sz))
        c0 += sz
    key = (device, tuple(q.shape), tuple(k.shape), q.dtype, tuple(sizes))
    st = _device_state(device, key, (BH, Lq, D), (BH, Lk, D), q.dtype)
    hq, hk, hv, ho = (t.view(BH, -1, D) for t in (q, k, v, out))
    compute = torch.cuda.current_stream(device)
    s_in, s_out = st["s_in"], st["s_out"]
    start = torch.cuda.Event()
    start.record(compute)
    for i, (c0, c1) in enumerate(chunks):
        # inputs of chunk i: after earlier work on the caller's stream and
        # after the previous call's attention read these device buffers
        s_in.wait_event(start)
        prev = st["done"].get(i)
        if prev is not None:
            s_in.wait_event(prev)
        with torch.cuda.stream(s_in):
            st["q"][c0:c1].copy_(hq[c0:c1], non_blocking=True)
            st["k"][c0:c1].copy_(hk[c0:c1], non_blocking=True)
            st["v"][c0:c1].copy_(hv[c0:c1], non_blocking=True)
        ready = torch.cuda.Event()
        ready.record(s_in)
        compute.wait_event(ready)
        o = attn_forward(st["q"][c0:c1].unsqueeze(0), st["k"][c0:c1].unsqueeze(0), st["v"][c0:c1].unsqueeze(0),
                         causal=causal, scale=scale)
        done = torch.cuda.Event()
        done.record(compute)
        st["done"][i] = done
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            ho[c0:c1].copy_(o[0], non_blocking=True)
        o.record_stream(s_out)
    compute.wait_stream(s_out)
    return out


__all__ = ["attn_forward_pinned", "MAX_CACHED_SHAPES"]
