"""Shared helpers for the parity tests (the oracle is the checker only)."""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "grouped-gemms_b200"))
sys.path.insert(0, ROOT)

from oracle import mx_oracle as O  # noqa: E402


def u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.uint8).cpu().numpy()


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 -> fp32 (round to nearest even)."""
    return O.bf16_bits_to_f32(O.f32_to_bf16_bits(np.ascontiguousarray(x, dtype=np.float32)))


def randn_bf16(shape, scale=1.0, seed=0, device="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(torch.bfloat16).to(device)


def as_oracle_input(t: torch.Tensor) -> np.ndarray:
    """Exact float32 values of a bf16/fp16/fp32 tensor."""
    return t.detach().float().cpu().numpy()


def quantize_ref(x: torch.Tensor):
    """Oracle quantisation of a torch tensor: (scales u8, e4m3 bytes)."""
    return O.to_mx(as_oracle_input(x))


def offsets(E, M, multiple_of=32, seed=0):
    import random
    rng = random.Random(seed)
    return O.generate_jagged_offs(E, M, multiple_of, rng=rng)


def gpu_status_clear():
    import mxgg
    return mxgg.device_status(clear=True)


def run_ranks(worker, world, *args, timeout=300):
    """Run `worker(rank, world, store, queue, *args)` in `world` spawned
    processes that rendezvous through a fresh file store (no TCP port to
    collide with another test's), and return {rank: message}."""
    import shutil
    import tempfile

    import torch.multiprocessing as mp
    d = tempfile.mkdtemp(prefix="mxgg_ranks_")
    store = os.path.join(d, "store")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=worker, args=(r, world, store, q) + tuple(args)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, msg = q.get(timeout=timeout)
            results[r] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
        shutil.rmtree(d, ignore_errors=True)
    return results


def blocked_scales_ref(s: np.ndarray, segments) -> np.ndarray:
    """CPU restatement of the blocked scale layout: the (R, C32) row-major
    e8m0 matrix `s` cut into row segments [(start, end), ...]; each segment's
    rows fill 128-row slabs of their own, slab j of a segment holding its rows
    128 j .. 128 j + 127; a slab is ceil(C32 / 4) atoms of 512 bytes, atom k4
    holding k-blocks 4 k4 .. 4 k4 + 3 of the slab's rows, row r, k-block k at
    byte (r % 32) * 16 + (r // 32) * 4 + k % 4.  Padding bytes are zero (as
    torch's to_blocked pads)."""
    R, C32 = s.shape
    cb = (C32 + 3) // 4
    slabs = sum((e - b + 127) // 128 for b, e in segments)
    out = np.zeros(slabs * cb * 512, dtype=np.uint8)
    slab0 = 0
    cols = np.arange(C32)
    for b, e in segments:
        rr = np.arange(e - b)
        if rr.size:
            slab = slab0 + rr // 128
            r128 = rr % 128
            idx = ((slab[:, None] * cb + cols[None, :] // 4) * 512 + (r128[:, None] % 32) * 16
                   + (r128[:, None] // 32) * 4 + cols[None, :] % 4)
            out[idx] = s[b:e]
        slab0 += (e - b + 127) // 128
    return out
