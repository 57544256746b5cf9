"""The reference's CPU path for the MXFP8 grouped GEMM, restated with torch
on the host cores (test and timing infrastructure only: bench.py's
``cpu_baseline`` and ``--impl reference`` legs time it, the CPU tests pin it;
no product path imports it).

The reference's GEMM kernels are Triton for gfx950 only; what of it runs on
a CPU is its quantiser ``to_mx`` (utils.py:67-105) and its offsets draw
(utils.py:35-50).  Its kernels compute ``out[g] = A[group g] @ B[g]^T``
(forward.py:485-488, forward and dgrad) and ``dW[g] = GO[group g]^T @
X[group g]`` (backward.py:230-231) on block-scaled e4m3 operands, whose exact
value is the dequantised product; so the CPU path is to_mx, dequantise
(x * 2^(s - 127) per 32-block) and a per-group fp32 torch.matmul.
``to_mx_cpu`` follows the reference's arithmetic in the same order -- fp32
block amax clamped to the smallest normal, the exponent taken from the fp32
bit pattern, scale = clamp(exponent - 8 + 127, 0, 254), divide, clamp to
+-448, round to e4m3 -- and is bit-exact with the reference's ``to_mx``
(pinned by tests/test_cpu_path.py against the golden vectors that
tests/golden/make_golden.py wrote from the reference's own function).
"""
import random
import time

import torch

BLOCK = 32
E4M3_MAX = 448.0
E4M3_MAX_POW2 = 8


def to_mx_cpu(x: torch.Tensor):
    """MXFP8 along the last dim: (scales uint8 (..., C/32), data float8_e4m3fn)."""
    shape = x.shape
    blocks = x.reshape(-1, shape[-1] // BLOCK, BLOCK)
    amax = blocks.abs().amax(dim=-1, keepdim=True).to(torch.float32)
    amax = amax.clamp(min=torch.finfo(torch.float32).tiny)
    exp = ((amax.view(torch.int32) >> 23) & 0xFF) - 127
    scale = (exp - E4M3_MAX_POW2 + 127).clamp(0, 254).to(torch.uint8)
    div = torch.exp2(scale.to(torch.float32) - 127)
    q = (blocks.to(torch.float32) / div).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return scale.reshape(*shape[:-1], shape[-1] // BLOCK), q.reshape(shape)


def dequant_cpu(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp32 values q * 2^(s - 127), one scale per 32 elements of the last dim."""
    shape = q.shape
    v = q.to(torch.float32).reshape(-1, shape[-1] // BLOCK, BLOCK)
    f = torch.exp2(s.to(torch.float32).reshape(-1, shape[-1] // BLOCK, 1) - 127)
    return (v * f).reshape(shape)


def grouped_mm_cpu(a: torch.Tensor, b: torch.Tensor, offs) -> torch.Tensor:
    """out[rows of group g] = a[rows] @ b[g]^T in fp32 (forward / dgrad)."""
    out = torch.zeros(a.shape[0], b.shape[1], dtype=torch.float32)
    start = 0
    for g, end in enumerate(offs):
        if end > start:
            out[start:end] = a[start:end] @ b[g].T
        start = end
    return out


def wgrad_cpu(go_t: torch.Tensor, ia_t: torch.Tensor, offs) -> torch.Tensor:
    """out[g] = go_t[:, group g] @ ia_t[:, group g]^T in fp32."""
    out = torch.zeros(len(offs), go_t.shape[0], ia_t.shape[0], dtype=torch.float32)
    start = 0
    for g, end in enumerate(offs):
        if end > start:
            out[g] = go_t[:, start:end] @ ia_t[:, start:end].T
        start = end
    return out


def draw_offs(E: int, M: int, multiple_of: int, rng: random.Random):
    """The reference bench's draw (utils.py:35-50): E-1 distinct multiples of
    `multiple_of` below M, sorted, then M."""
    vals = list(range(multiple_of, M + 1, multiple_of))
    return sorted(rng.sample(vals[:-1], E - 1) + [M])


class CpuPathSample:
    """A bounded sample of the 36-shape sweep through the reference's CPU path:
    every timed point quantises its bf16 operands with to_mx, dequantises and
    runs the per-group fp32 matmuls, at the sweep's full M = 16640 tokens.
    Points are (shape, pass) pairs over `shapes`; `run_point(i)` times one."""

    SHAPES = [(1, 2048, 2048), (2, 5120, 5120), (8, 2048, 2048), (8, 8192, 2048)]
    PASSES = ("fwd", "dgrad", "wgrad")
    M = 16640

    def __init__(self, threads=None, seed=123, shapes=None, M=None):
        if threads:
            torch.set_num_threads(int(threads))
        self.threads = torch.get_num_threads()
        self.shapes = list(shapes or self.SHAPES)
        self.M = int(M or self.M)
        rng = random.Random(seed)
        gen = torch.Generator().manual_seed(seed)
        self.points = []
        for (E, N, K) in self.shapes:
            offs = draw_offs(E, self.M, 32, rng)
            for p in self.PASSES:
                self.points.append((p, (E, N, K), offs))
        self._gen = gen

    def describe(self) -> str:
        return (f"reference CPU path (to_mx of both bf16 operands + dequantise + per-group fp32 torch.matmul) "
                f"at M={self.M} tokens on {len(self.points)} (shape, pass) points: (E, N, K) in {self.shapes} x "
                f"{'/'.join(self.PASSES)}; geomean of per-point TFLOPS, {self.threads} threads")

    def _operands(self, pass_, E, N, K):
        g, M = self._gen, self.M
        if pass_ == "fwd":
            return (torch.randn(M, K, generator=g).to(torch.bfloat16),
                    torch.randn(E, N, K, generator=g).to(torch.bfloat16))
        if pass_ == "dgrad":
            return (torch.randn(M, N, generator=g).to(torch.bfloat16),
                    torch.randn(E, K, N, generator=g).to(torch.bfloat16))
        return (torch.randn(N, M, generator=g).to(torch.bfloat16),
                torch.randn(K, M, generator=g).to(torch.bfloat16))

    def run_point(self, i: int) -> float:
        """TFLOPS of point i (to_mx, dequantise and matmul inside the timing)."""
        pass_, (E, N, K), offs = self.points[i % len(self.points)]
        a, b = self._operands(pass_, E, N, K)
        t0 = time.perf_counter()
        a_s, a_q = to_mx_cpu(a)
        b_s, b_q = to_mx_cpu(b)
        ad, bd = dequant_cpu(a_q, a_s), dequant_cpu(b_q, b_s)
        if pass_ == "wgrad":
            wgrad_cpu(ad, bd, offs)
        else:
            grouped_mm_cpu(ad, bd, offs)
        dt = time.perf_counter() - t0
        return 2.0 * self.M * N * K / dt / 1e12
