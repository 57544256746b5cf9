"""mxgg_pack_a_atoms_multi (one launch for every destination of an
expert-parallel sender) writes the same bytes as one mxgg_pack_a_atoms call
per destination, including packs with no rows and segments shorter than a
128-row slab."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_multi_pack_equals_single_packs():
    from mxgg import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    K = 1280                                   # 10 stages: a partial 4-stage chunk
    rows_total = 3000
    g = torch.Generator(device=dev).manual_seed(3)
    a_s = torch.randint(0, 256, (rows_total, K // 32), generator=g, device=dev, dtype=torch.int32).to(torch.uint8)
    # (first row, segment lengths) of each destination's rows
    packs = [(0, [100, 0, 700]), (800, []), (800, [129, 1, 1000]), (1930, [1070])]
    slab_bytes = (K + 127) // 128 * 512
    singles, multis, cums = [], [], []
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for first, segs in packs:
        rows = sum(segs)
        cum = torch.tensor(segs or [0], dtype=torch.int64).cumsum(0).to(torch.int32).to(dev)
        cums.append(cum)
        n_slabs = sum((c + 127) // 128 for c in segs) + 1
        a = torch.full((n_slabs * slab_bytes,), 0xAB, dtype=torch.uint8, device=dev)
        b = a.clone()
        singles.append(a)
        multis.append(b)
        if rows:
            _lib.check(lib.mxgg_pack_a_atoms(ctypes.c_void_p(a_s.data_ptr() + first * (K // 32)),
                                             ctypes.c_void_p(cum.data_ptr()), rows, K, cum.numel(),
                                             ctypes.c_void_p(a.data_ptr()), stream), "mxgg_pack_a_atoms")
    n = len(packs)
    i64 = ctypes.c_int64 * n
    vp = ctypes.c_void_p * n
    _lib.check(lib.mxgg_pack_a_atoms_multi(ctypes.c_void_p(a_s.data_ptr()), K, n,
                                           i64(*[f for f, _ in packs]), i64(*[sum(s) for _, s in packs]),
                                           vp(*[c.data_ptr() for c in cums]), i64(*[c.numel() for c in cums]),
                                           vp(*[m.data_ptr() for m in multis]), stream),
               "mxgg_pack_a_atoms_multi")
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(singles, multis)):
        assert torch.equal(a, b), f"pack {i} differs"
    assert not torch.equal(singles[0], torch.full_like(singles[0], 0xAB))   # the packs wrote something
