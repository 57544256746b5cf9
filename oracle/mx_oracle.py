"""CPU oracle for the MXFP8 grouped-GEMM hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The library under ``grouped-gemms_b200/``
never imports it and has no CPU fallback.

It restates, in numpy, the arithmetic of the reference repository
(indianspeedster/grouped-gemms) for the three passes of the path:

* ``to_mx``            -- ``utils.py:67-105`` (FLOOR-mode MXFP8 quantiser)
* ``grouped_mm``       -- ``kernels/forward.py:485-497`` semantics of
                          ``triton_mxfp8_grouped_mm``: per group
                          ``deq(A_g) @ deq(B_g)^T`` with fp32 accumulation
                          (``forward.py:211,238-240``) and a cast of the
                          accumulator to ``out_dtype`` (``forward.py:293``)
* ``wgrad``            -- ``kernels/backward.py:230-244``: per group
                          ``deq(GO_g)^T @ deq(X_g)`` where the jagged token
                          dimension is the contraction and the e8m0 scales run
                          along tokens (``backward.py:81-98``)
* ``build_tile_map``   -- ``kernels/forward.py:296-365`` (``_expt_data_kernel``
                          / ``_build_expt_data``): per-group histogram, start
                          offsets, padded tile count and the packed
                          ``(block << 16) | expert`` map, ``-1`` padded.
* ``compute_error``    -- ``test_correctness.py:20-23`` (SQNR in dB).

Pinning: ``to_mx`` and ``generate_jagged_offs`` are checked bit-for-bit
against vectors produced by the reference's own functions
(``tests/golden/make_golden.py``).  The GEMM emulation is checked against the
reference-style torch emulation (dequantise, fp32 matmul per group) stored in
the same fixtures.  The routing map has no runnable reference (Triton/ROCm
only), so its restatement is pinned only by reading ``forward.py:312-338``.
"""

from __future__ import annotations

import random

import numpy as np

# e4m3fn constants (utils.py:62-64): max finite 448 = 1.75 * 2**8.
E4M3_MAX = 448.0
E4M3_MAX_POW2 = 8
# e2m1 (MXFP4) constants: max finite 6 = 1.5 * 2**2.  The reference has no
# fp4 path; FLOOR mode is extended by analogy (emax = 2).
E2M1_MAX = 6.0
E2M1_MAX_POW2 = 2
BLOCK = 32


# ---------------------------------------------------------------------------
# bit helpers
# ---------------------------------------------------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 values (exact widening)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits with round-to-nearest-even (torch's ``.to(bf16)``)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def e4m3_encode(v: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn bytes, round-to-nearest-even.

    Restates torch's float->float8_e4m3fn cast as used by ``utils.py:101``.
    Inputs are already clamped to [-448, 448] by the reference, so no
    saturation step is needed; NaN keeps its sign (0x7F / 0xFF), matching the
    CPU cast.
    """
    v = np.asarray(v, dtype=np.float32)
    sign = (v.view(np.uint32) >> 31).astype(np.uint8)
    a = np.abs(v.astype(np.float64))
    out = np.zeros(v.shape, dtype=np.uint8)
    nan = np.isnan(v)
    with np.errstate(invalid="ignore"):
        sub = a < 2.0 ** -6
    # subnormal range: step 2**-9; rounding up to 8 gives the min normal 0x08
    ms = np.rint(np.where(sub, a, 0.0) * 2.0 ** 9).astype(np.int64)
    enc_sub = ms
    # normal range
    an = np.where(sub | nan, 1.0, a)
    m, e = np.frexp(an)               # an = m * 2**e, m in [0.5, 1)
    e = e - 1                         # an = (2m) * 2**e, 2m in [1, 2)
    frac = np.rint((2.0 * m - 1.0) * 8.0).astype(np.int64)
    carry = frac == 8
    frac = np.where(carry, 0, frac)
    e = e + carry
    enc_norm = ((e + 7) << 3) | frac
    enc = np.where(sub, enc_sub, enc_norm)
    out[...] = np.clip(enc, 0, 0x7E).astype(np.uint8)
    out |= (sign << 7)
    out[nan] = np.where(sign[nan] == 1, 0xFF, 0x7F).astype(np.uint8)
    return out


_E4M3_TABLE = None


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    """e4m3fn bytes -> float32 values (exact)."""
    global _E4M3_TABLE
    if _E4M3_TABLE is None:
        t = np.zeros(256, dtype=np.float32)
        for i in range(256):
            s = -1.0 if i & 0x80 else 1.0
            e = (i >> 3) & 0xF
            m = i & 7
            if e == 0xF and m == 7:
                t[i] = np.nan
            elif e == 0:
                t[i] = s * m * 2.0 ** -9
            else:
                t[i] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
        _E4M3_TABLE = t
    return _E4M3_TABLE[np.asarray(b, dtype=np.uint8)]


_E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float64)


def e2m1_encode(v: np.ndarray) -> np.ndarray:
    """float32 (already clamped to [-6, 6]) -> e2m1 nibbles, RNE on the grid.

    e2m1 has no NaN: NaN becomes +6 (code 0b0111), the rule of the hardware
    conversion the GPU quantiser uses.  (MXFP4 has no reference
    implementation; this defines it.)"""
    v = np.asarray(v, dtype=np.float32)
    nan = np.isnan(v)
    sign = (v.view(np.uint32) >> 31).astype(np.uint8)
    a = np.abs(v.astype(np.float64))
    # grid points 0,.5,1,1.5,2,3,4,6 ; ties go to the even mantissa code
    codes = np.zeros(v.shape, dtype=np.uint8)
    for c in range(1, 8):
        lo, hi = _E2M1_VALUES[c - 1], _E2M1_VALUES[c]
        mid = 0.5 * (lo + hi)
        # ties-to-even: code c-1 is even when (c-1) % 2 == 0
        if (c - 1) % 2 == 0:
            up = a > mid
        else:
            up = a >= mid
        codes = np.where(up, c, codes).astype(np.uint8)
    out = codes | (sign << 3)
    return np.where(nan, np.uint8(7), out).astype(np.uint8)


def pack_e2m1(nibbles: np.ndarray) -> np.ndarray:
    """(..., 2n) nibbles -> (..., n) bytes, element 2i in the low nibble."""
    n = np.asarray(nibbles, dtype=np.uint8)
    return (n[..., 0::2] & 0xF) | ((n[..., 1::2] & 0xF) << 4)


def unpack_e2m1(packed: np.ndarray) -> np.ndarray:
    """(..., n) bytes -> (..., 2n) nibbles (inverse of pack_e2m1)."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (2 * p.shape[-1],), dtype=np.uint8)
    out[..., 0::2] = p & 0xF
    out[..., 1::2] = p >> 4
    return out


def e2m1_decode(n: np.ndarray) -> np.ndarray:
    n = np.asarray(n, dtype=np.uint8)
    s = np.where(n & 8, -1.0, 1.0)
    return (s * _E2M1_VALUES[n & 7]).astype(np.float32)


# ---------------------------------------------------------------------------
# to_mx  (utils.py:67-105)
# ---------------------------------------------------------------------------

def to_mx(x: np.ndarray, block: int = BLOCK, elem: str = "e4m3"):
    """FLOOR-mode MX quantisation along the last dim.

    ``x`` holds float32 values (widened from the caller's bf16/fp16/fp32).
    Returns ``(scales_u8, data)`` -- scales first, like ``utils.py:105``.
    ``data`` is e4m3 bytes for ``elem='e4m3'`` or e2m1 nibbles (one per
    byte, unpacked) for ``elem='e2m1'``.

    Steps (utils.py:86-101):
      amax over the 32-block (NaN propagates, utils.py:86)
      clamp(amax, FLT_MIN)                                   (utils.py:88)
      e = biased exponent of amax; s = clamp(e - 127 - emax + 127, 0, 254)
      q = cast(clamp(x / 2**(s-127), -max, max))
    """
    x = np.asarray(x, dtype=np.float32)
    assert x.shape[-1] % block == 0
    lead = x.shape[:-1]
    xb = x.reshape(-1, x.shape[-1] // block, block)
    absbits = xb.view(np.uint32) & 0x7FFFFFFF
    amax_bits = absbits.max(axis=-1)          # NaN bit patterns sort above inf
    amax_bits = np.maximum(amax_bits, 0x00800000)   # clamp(min=FLT_MIN)
    exp = ((amax_bits >> 23) & 0xFF).astype(np.int64) - 127
    emax = E4M3_MAX_POW2 if elem == "e4m3" else E2M1_MAX_POW2
    s = np.clip(exp - emax + 127, 0, 254).astype(np.uint8)
    scale = np.exp2(s.astype(np.float64) - 127.0)
    vmax = E4M3_MAX if elem == "e4m3" else E2M1_MAX
    with np.errstate(invalid="ignore", over="ignore"):
        q = (xb.astype(np.float64) / scale[..., None]).astype(np.float32)
        q = np.where(np.isnan(q), q, np.clip(q, -vmax, vmax)).astype(np.float32)
    # the division keeps the NaN sign on the CPU path
    q = np.where(np.isnan(xb), xb, q)
    data = e4m3_encode(q) if elem == "e4m3" else e2m1_encode(q)
    return s.reshape(*lead, x.shape[-1] // block), data.reshape(x.shape)


def dequant(data: np.ndarray, scales: np.ndarray, block: int = BLOCK,
            elem: str = "e4m3") -> np.ndarray:
    """``data * 2**(scale - 127)`` per 32-block along the last dim (float64)."""
    v = e4m3_decode(data) if elem == "e4m3" else e2m1_decode(data)
    v = v.astype(np.float64).reshape(*data.shape[:-1], data.shape[-1] // block, block)
    sc = np.exp2(scales.astype(np.float64) - 127.0)
    return (v * sc[..., None]).reshape(data.shape)


# ---------------------------------------------------------------------------
# grouped GEMMs
# ---------------------------------------------------------------------------

def group_bounds(offs, M: int):
    """(start, end) per group from cumulative ends (forward.py:321-325)."""
    offs = [int(o) for o in np.asarray(offs).tolist()]
    out, prev = [], 0
    for o in offs:
        out.append((prev, o))
        prev = o
    return out


def grouped_mm(a_q, a_s, b_q, b_s, offs, acc=np.float64,
               a_elem="e4m3", b_elem="e4m3"):
    """fp32 result of ``triton_mxfp8_grouped_mm`` (forward.py:485-497).

    a_q (M,K) bytes, a_s (M,K/32); b_q (E,N,K), b_s (E,N,K/32).  Rows of the
    output past ``offs[-1]`` are returned as NaN: the reference leaves them
    uninitialised (forward.py:583), so tests must not compare them.
    """
    M, K = a_q.shape
    E, N, _ = b_q.shape
    A = dequant(a_q, a_s, elem=a_elem).astype(acc)
    out = np.full((M, N), np.nan, dtype=np.float32)
    for g, (s, e) in enumerate(group_bounds(offs, M)):
        if e <= s:
            continue
        B = dequant(b_q[g], b_s[g], elem=b_elem).astype(acc)
        out[s:e] = (A[s:e] @ B.T).astype(np.float32)
    return out


def wgrad(go_t_q, go_s, ia_t_q, ia_s, offs, acc=np.float64):
    """fp32 result of ``triton_mxfp8_wgrad`` (backward.py:230-305).

    go_t_q (N,M) bytes with go_s (N,M/32); ia_t_q (K,M) with ia_s (K,M/32).
    Returns (E,N,K): ``dW[g] = sum_{m in group g} deq(go)[n,m] * deq(ia)[k,m]``.
    Empty groups give zeros (the reference's loop runs zero times,
    backward.py:67, and stores the zero accumulator).
    """
    N, M = go_t_q.shape
    K = ia_t_q.shape[0]
    GO = dequant(go_t_q, go_s).astype(acc)
    IA = dequant(ia_t_q, ia_s).astype(acc)
    E = len(offs)
    out = np.zeros((E, N, K), dtype=np.float32)
    for g, (s, e) in enumerate(group_bounds(offs, M)):
        if e > s:
            out[g] = (GO[:, s:e] @ IA[:, s:e].T).astype(np.float32)
    return out


def build_tile_map(offs, M: int, block_m: int):
    """Restatement of ``_expt_data_kernel`` (forward.py:312-338).

    Returns (hist, offs_raw, offs_pad_sum, block_pid_map) where
    block_pid_map has ``cdiv(M, block_m) + max(E-1, 0)`` entries
    (forward.py:347) holding ``(block << 16) | expert`` or -1.
    """
    offs = [int(o) for o in np.asarray(offs).tolist()]
    E = len(offs)
    grid_m_ub = -(-M // block_m) + max(E - 1, 0)
    hist, offs_raw, blocks = [], [], []
    prev = 0
    for o in offs:
        h = o - prev
        hist.append(h)
        offs_raw.append(prev)
        blocks.append((h + block_m - 1) // block_m)
        prev = o
    pid_map = []
    for pid in range(grid_m_ub):
        cum, val = 0, -1
        for e in range(E):
            nxt = cum + blocks[e]
            if cum <= pid < nxt:
                val = ((pid - cum) << 16) | e
            cum = nxt
        pid_map.append(val)
    return (np.array(hist, np.int32), np.array(offs_raw, np.int32),
            np.int32(sum(blocks)), np.array(pid_map, np.int32))


def compute_error(x: np.ndarray, y: np.ndarray) -> float:
    """SQNR in dB (test_correctness.py:20-23)."""
    x = np.asarray(x, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    return float(20.0 * np.log10(np.linalg.norm(x) / np.linalg.norm(x - y)))


def rel_l2(x: np.ndarray, ref: np.ndarray) -> float:
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / (d if d > 0 else 1.0))


# ---------------------------------------------------------------------------
# seeded fixtures (utils.py:35-50, bench.py:113-122, 243-257)
# ---------------------------------------------------------------------------

def generate_jagged_offs(E: int, M: int, multiple_of: int = 32, rng=random):
    """Same draw as ``utils.generate_jagged_offs`` (Python ``random.sample``)."""
    if M % multiple_of != 0:
        raise ValueError(f"M must be divisible by {multiple_of}")
    possible = list(range(multiple_of, M + 1, multiple_of))
    if E > len(possible):
        raise ValueError("E cannot be larger than the number of possible values")
    sel = rng.sample(possible[:-1], E - 1)
    return np.array(sorted(sel + [M]), dtype=np.int32)


def llama4_shapes():
    """The 36 (E, M, N, K) shapes in the reference's order (bench.py:113-122)."""
    out = []
    for e in (1, 2, 4, 8):
        for n in (2048, 5120, 8192):
            for k in (2048, 5120, 8192):
                out.append((e, 16640, n, k))
    return out


def llama4_offsets(seed: int = 123):
    """Offsets drawn exactly as the reference bench does (bench.py:250-256)."""
    rng = random.Random(seed)
    return [generate_jagged_offs(e, m, 32, rng=rng) for (e, m, n, k) in llama4_shapes()]
