"""Generate the committed golden fixtures from the reference's own code.

Run from the repository root in a container that has the reference checkout::

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's ``utils.to_mx`` and ``utils.generate_jagged_offs``
(``utils.py:35-105``) unchanged and records their outputs.  The GEMM
fixtures hold the reference-style emulation used by torchao's and the
reference's tests: quantise with the reference ``to_mx``, dequantise, then a
per-group fp32 ``torch.matmul`` (``test_correctness.py:36-50`` quantisation,
``forward.py:485-497`` / ``backward.py:230-244`` semantics).  The reference's
Triton kernels are ROCm-only and cannot run here, so that emulation is the
strongest pin available for the GEMM passes.

Outputs (``tests/golden/*.npz``) are small and deterministic; the GPU box
never needs the reference checkout.
"""

import os
import random
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _bits32(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int32).numpy().view(np.uint32)


def _u8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy()


def _deq(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    v = q.to(torch.float32)
    sh = v.shape
    v = v.reshape(*sh[:-1], sh[-1] // 32, 32)
    sc = torch.exp2(s.to(torch.float32) - 127.0)
    return (v * sc[..., None]).reshape(sh)


def to_mx_edge_inputs() -> dict:
    """fp32 blocks that exercise every branch of utils.py:86-101."""
    blocks = []
    z = np.zeros(32, np.float32)
    blocks.append(z.copy())                                   # all zero -> scale 0
    b = z.copy(); b[3] = np.inf; b[4] = 1.0; blocks.append(b)   # +inf
    b = z.copy(); b[7] = -np.inf; b[8] = -3.0; blocks.append(b)  # -inf
    b = z.copy(); b[1] = np.nan; b[2] = 5.0; blocks.append(b)   # +nan
    nb = np.array([0xFFC00000], np.uint32).view(np.float32)[0]
    b = z.copy(); b[9] = nb; b[10] = -2.0; blocks.append(b)     # -nan
    for p in (-126, -120, -10, -1, 0, 1, 8, 9, 100, 127):       # amax an exact power of two
        b = np.linspace(-1, 1, 32).astype(np.float32) * np.float32(2.0 ** p)
        blocks.append(b)
    for v in (448.0, 464.0, 479.9, 480.0, 500.0, 1e-3, 2.0 ** -130, 2.0 ** -149):
        b = np.full(32, v, np.float32); b[::2] *= -1; blocks.append(b)
    # e4m3 subnormal outputs: a large value next to tiny ones
    b = (np.arange(32, dtype=np.float32) * np.float32(2.0 ** -9)); b[0] = 448.0; blocks.append(b)
    b = (np.arange(32, dtype=np.float32) * np.float32(0.37)) * np.float32(2.0 ** -12); b[31] = 1.0; blocks.append(b)
    # ties for round-to-nearest-even in e4m3
    b = np.array([1.0 + k / 16.0 for k in range(32)], np.float32); blocks.append(b)
    b = np.array([(2 * k + 1) * 2.0 ** -10 for k in range(32)], np.float32); b[31] = 256.0; blocks.append(b)
    # fp32 subnormal inputs
    b = (np.arange(1, 33, dtype=np.float32) * np.float32(2.0 ** -140)); blocks.append(b)
    return np.stack(blocks).astype(np.float32)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from utils import generate_jagged_offs, to_mx  # the reference's own helpers

    out = {}

    # ---- to_mx: seeded bf16 randn (the GEMM inputs' distribution) ----------
    torch.manual_seed(0)
    x = torch.randn(64, 256, dtype=torch.bfloat16)
    x[5] *= 1000.0
    x[6] *= 1e-3
    s, q = to_mx(x)
    out["tomx_bf16_x"] = _bits16(x)
    out["tomx_bf16_s"] = _u8(s)
    out["tomx_bf16_q"] = _u8(q)

    # ---- to_mx: fp32 edge blocks --------------------------------------------
    xe = torch.from_numpy(to_mx_edge_inputs())
    s, q = to_mx(xe)
    out["tomx_edge_x"] = _bits32(xe)
    out["tomx_edge_s"] = _u8(s)
    out["tomx_edge_q"] = _u8(q)

    # ---- to_mx: 3-D fp32 input, wide dynamic range ----------------------------
    torch.manual_seed(1)
    x3 = torch.randn(3, 17, 96, dtype=torch.float32) * torch.exp2(torch.randint(-30, 30, (3, 17, 1)).float())
    s, q = to_mx(x3)
    out["tomx_f32_x"] = _bits32(x3)
    out["tomx_f32_s"] = _u8(s)
    out["tomx_f32_q"] = _u8(q)

    # ---- generate_jagged_offs: the reference bench's exact sequence -------------
    random.seed(123)
    offs = []
    for e in (1, 2, 4, 8):
        for n in (2048, 5120, 8192):
            for k in (2048, 5120, 8192):
                offs.append(generate_jagged_offs(e, 16640, multiple_of=32, device="cpu").numpy())
    out["llama4_offs"] = np.concatenate(offs).astype(np.int32)
    out["llama4_offs_lens"] = np.array([len(o) for o in offs], np.int32)

    # ---- forward config 1 (CPU-runnable small case) -----------------------------
    random.seed(0)
    torch.manual_seed(0)
    E, M, N, K = 4, 1024, 256, 512
    A = torch.randn(M, K, dtype=torch.bfloat16)
    B = torch.randn(E, N, K, dtype=torch.bfloat16) * 0.02
    offs1 = generate_jagged_offs(E, M, multiple_of=32, device="cpu")
    a_s, a_q = to_mx(A)
    b_s, b_q = to_mx(B)
    Ad, Bd = _deq(a_q, a_s), _deq(b_q, b_s)
    ref = torch.full((M, N), float("nan"))
    prev = 0
    for g in range(E):
        end = int(offs1[g])
        ref[prev:end] = Ad[prev:end] @ Bd[g].t()
        prev = end
    hp = torch._grouped_mm(A, B.transpose(-2, -1), offs=offs1, out_dtype=torch.bfloat16)
    out.update({
        "fwd1_a_bits": _bits16(A), "fwd1_b_bits": _bits16(B),
        "fwd1_a_q": _u8(a_q), "fwd1_a_s": _u8(a_s),
        "fwd1_b_q": _u8(b_q), "fwd1_b_s": _u8(b_s),
        "fwd1_offs": offs1.numpy().astype(np.int32),
        "fwd1_out_f32": ref.numpy().astype(np.float32),
        "fwd1_hp_bf16": _bits16(hp),
    })

    # ---- wgrad small case: dim1-quantised (scales along tokens) -----------------
    random.seed(1)
    torch.manual_seed(2)
    E, M, N, K = 3, 512, 128, 256
    go = torch.randn(M, N, dtype=torch.bfloat16)
    xx = torch.randn(M, K, dtype=torch.bfloat16)
    offsw = generate_jagged_offs(E, M, multiple_of=32, device="cpu")
    go_s, go_q = to_mx(go.t().contiguous())     # (N, M/32), (N, M)
    ia_s, ia_q = to_mx(xx.t().contiguous())     # (K, M/32), (K, M)
    God, Iad = _deq(go_q, go_s), _deq(ia_q, ia_s)
    refw = torch.zeros(E, N, K)
    prev = 0
    for g in range(E):
        end = int(offsw[g])
        refw[g] = God[:, prev:end] @ Iad[:, prev:end].t()
        prev = end
    out.update({
        "wg_go_q": _u8(go_q), "wg_go_s": _u8(go_s),
        "wg_ia_q": _u8(ia_q), "wg_ia_s": _u8(ia_s),
        "wg_offs": offsw.numpy().astype(np.int32),
        "wg_out_f32": refw.numpy().astype(np.float32),
    })

    path = os.path.join(HERE, "golden_v1.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
