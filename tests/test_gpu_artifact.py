"""Packed trellis rows on the GPU against the reference's own encode_entry / decode_rotated output (tests/golden/
artifact.npz, made by make_golden.py from compiler_artifact.py) and the oracle's pack_trellis (compiler_artifact.py:
225-297): bit-exact words, states and decoded values; the product against a dense fp64 product."""

import numpy as np
import pytest
import torch

import oracle.core as O

pytestmark = pytest.mark.gpu


def _u32(t):
    return t.cpu().numpy().view(np.uint32)


def _path(rows, n, k, seed, L=12):
    """Random trellis paths from state 0: each state shifts the previous one by k bits and appends a symbol."""
    rng = np.random.default_rng(seed)
    sym = rng.integers(0, 1 << k, size=(rows, n))
    st = np.zeros((rows, n), dtype=np.int64)
    s = np.zeros(rows, dtype=np.int64)
    for j in range(n):
        s = ((s << k) | sym[:, j]) & ((1 << L) - 1)
        st[:, j] = s
    return st


def test_pack_unpack_match_reference_groups(golden):
    from lookatmyquant_b200 import artifact as A
    g = golden("artifact")
    for i in range(4):
        rows, bits = g[f"g{i}_rows"].astype(np.int64), int(g[f"g{i}_bits"])
        ti = int(g["states"][rows[0], 0]) // 4096
        states = torch.as_tensor(g["states"][rows].astype(np.int64) - 4096 * ti).cuda()
        codes = A.pack_trellis(states, bits)
        assert np.array_equal(_u32(codes), g[f"g{i}_codes"])
        back = A.unpack_trellis(codes, bits, 200)
        assert np.array_equal(back.cpu().numpy().astype(np.int64), states.cpu().numpy())


def test_encode_entry_and_decode_rotated_match_reference(golden):
    from lookatmyquant_b200 import artifact as A
    g = golden("artifact")
    perm_rows = [torch.as_tensor(g[f"g{i}_rows"].astype(np.int64)) for i in range(4)]
    bits = [int(g[f"g{i}_bits"]) for i in range(4)]
    entry = {"states": torch.as_tensor(g["states"]).cuda(), "scales": torch.as_tensor(g["scales"]),
             "in_seed": int(g["in_seed"]), "table": torch.as_tensor(g["table"]),
             "row_groups": [{"rows": r, "bits": b, "table_index": i} for i, (r, b) in enumerate(zip(perm_rows, bits))]}
    tensors, meta = A.encode_entry("w", entry)
    assert np.array_equal(tensors["w.signs"].numpy(), g["signs"])
    for i in range(4):
        assert np.array_equal(_u32(tensors[f"w.g{i}.rows"]), g[f"g{i}_rows"])
        assert np.array_equal(_u32(tensors[f"w.g{i}.codes"]), g[f"g{i}_codes"])
        assert np.array_equal(tensors[f"w.g{i}.scales"].cpu().numpy(), g[f"g{i}_scales"])
    assert [gr["bits"] for gr in meta["groups"]] == bits and meta["shape"] == [200, 200]
    dec = A.decode_rotated(tensors, meta)
    assert np.array_equal(dec.cpu().numpy(), g["decoded"])


@pytest.mark.parametrize("k", [1, 2, 3, 4])
@pytest.mark.parametrize("n", [1, 31, 32, 200, 2560 + 7])
def test_pack_matches_oracle_on_random_paths(k, n):
    from lookatmyquant_b200 import artifact as A
    st = _path(37, n, k, 100 * k + n)
    codes = A.pack_trellis(torch.as_tensor(st).cuda(), k)
    assert np.array_equal(_u32(codes), O.pack_trellis(st, k))
    assert np.array_equal(A.unpack_trellis(codes, k, n).cpu().numpy().astype(np.int64), st)


def test_pack_rejects_a_broken_path():
    from lookatmyquant_b200 import artifact as A
    st = _path(4, 100, 2, 1)
    st[2, 50] ^= 1 << 11  # the state's high bits no longer continue the previous state
    with pytest.raises(ValueError, match="not a row trellis from zero"):
        A.pack_trellis(torch.as_tensor(st).cuda(), 2)
    st = _path(4, 100, 2, 2)
    st[1, 0] = 5  # the first state must come from state 0
    with pytest.raises(ValueError, match="not a row trellis from zero"):
        A.pack_trellis(torch.as_tensor(st).cuda(), 2)


@pytest.mark.parametrize("nvec", [1, 3, 16, 21, 64])
def test_product_matches_dense(golden, nvec):
    from lookatmyquant_b200 import artifact as A
    from lookatmyquant_b200.rotation import Rotation
    g = golden("artifact")
    tensors = {"w.signs": torch.as_tensor(g["signs"])}
    groups = []
    for i in range(4):
        key = f"w.g{i}"
        tensors.update({key + ".rows": torch.as_tensor(g[f"g{i}_rows"].view(np.int32)).cuda(),
                        key + ".codes": torch.as_tensor(g[f"g{i}_codes"].view(np.int32)).cuda(),
                        key + ".scales": torch.as_tensor(g[f"g{i}_scales"]).cuda()})
        ti = int(g["states"][int(g[f"g{i}_rows"][0]), 0]) // 4096
        tensors[key + ".table"] = torch.as_tensor(g["table"][4096 * ti:4096 * (ti + 1)]).cuda()
        groups.append({"rows": len(g[f"g{i}_rows"]), "bits": int(g[f"g{i}_bits"])})
    meta = A.grouped_matrix_meta("w", [200, 200], groups)
    prod = A.TrellisProduct(tensors, meta)
    x = torch.randn(nvec, 200, dtype=torch.float64, generator=torch.Generator().manual_seed(nvec)).cuda()
    y = prod(x).double().cpu().numpy()
    xr = Rotation.from_signs(torch.as_tensor(g["signs"]).double()).rows(x).cpu().numpy()
    ref = xr @ g["decoded"].astype(np.float64).T
    tol = 1e-2 if nvec >= A.GEMM_PRODUCT_VECTORS else 1e-5  # bf16 tensor-core GEMM vs the fp32 packed product
    assert np.abs(y - ref).max() <= tol * np.abs(ref).max()


def _random_product(m, n, widths, seed, name="w"):
    """A grouped matrix of m rows whose row groups have the given symbol widths (random rows, valid paths, a random
    4096-entry table each)."""
    from lookatmyquant_b200 import artifact as A
    gen = torch.Generator().manual_seed(seed)
    perm = torch.randperm(m, generator=gen)
    cuts = np.linspace(0, m, len(widths) + 1).astype(int)
    tensors = {name + ".signs": A.input_signs(n, seed)}
    groups = []
    for i, k in enumerate(widths):
        rows = perm[cuts[i]:cuts[i + 1]].sort().values
        key = f"{name}.g{i}"
        states = torch.as_tensor(_path(rows.numel(), n, k, seed + i)).cuda()
        tensors.update({key + ".rows": rows.to(torch.int32).cuda(), key + ".codes": A.pack_trellis(states, k),
                        key + ".scales": (0.5 + torch.rand(rows.numel(), generator=gen)).float().cuda(),
                        key + ".table": torch.randn(4096, generator=gen).float().cuda()})
        groups.append({"rows": rows.numel(), "bits": k})
    return A.TrellisProduct(tensors, A.grouped_matrix_meta(name, [m, n], groups))


def _per_group(prod, xr):
    """The product with one lamq_trellis_product launch per row group (the per-group kernel)."""
    from lookatmyquant_b200 import _lib
    from lookatmyquant_b200._lib import check, ptr, stream_ptr
    lib = _lib.load()
    y = torch.full((xr.shape[0], prod.m), float("nan"), device="cuda")
    for g, codes, rows, scales, table in prod.groups:
        check(lib.lamq_trellis_product(ptr(codes), rows.numel(), prod.n, g["bits"], g["state_bits"], ptr(scales),
                                       ptr(table), ptr(rows), ptr(xr), xr.stride(0), xr.shape[0], ptr(y), y.stride(0),
                                       stream_ptr(y.device)), "lamq_trellis_product")
    return y


@pytest.mark.parametrize("n", [284, 4352])
@pytest.mark.parametrize("nvec", [1, 5, 21])
def test_grouped_product_equals_per_group_launches(nvec, n):
    """lamq_trellis_product_groups over a stage (three matrices, 1-4-bit groups and a 6-bit one, 39 row groups: two
    launches of at most 32) gives every row exactly the per-group kernel's value, for aligned and unaligned inputs.
    n = 284: two 256-column blocks, the last one ragged (n is 4 mod 8); n = 4352: 17 blocks, so warps take several."""
    from lookatmyquant_b200 import artifact as A
    prods = [_random_product(300, n, [1, 2, 3, 4] * 3, 11), _random_product(77, n, [2, 4, 6], 12, "v"),
             _random_product(130, n, [4, 3, 2, 1] * 6, 13, "u")]
    gen = torch.Generator().manual_seed(nvec)
    base = torch.randn(nvec, n + 1, generator=gen).float().cuda()
    for xr in (base[:, :n].contiguous(), base[:, 1:]):  # 16-byte rows, then rows at an odd offset and stride
        ys = A.product_rotated(prods, xr)
        for p, y in zip(prods, ys):
            ref = _per_group(p, xr)
            assert not torch.isnan(ref).any()
            assert torch.equal(y, ref)
            assert torch.equal(p.rotated(xr), ref)


def test_grouped_product_skips_empty_groups():
    from lookatmyquant_b200 import _lib
    from lookatmyquant_b200._lib import check, ptr, stream_ptr
    p = _random_product(40, 64, [3, 1], 5)
    xr = torch.randn(2, 64).float().cuda()
    y = torch.zeros(2, 40, device="cuda")
    (g0, _), (g1, _) = p.product_groups(y)
    empty = _lib.ProductGroup(None, 0, 2, 12, None, None, None, None, 0)
    arr = (_lib.ProductGroup * 4)(empty, g0, empty, g1)
    check(_lib.load().lamq_trellis_product_groups(arr, 4, 64, ptr(xr), 64, 2, stream_ptr()), "groups")
    assert torch.equal(y, _per_group(p, xr))


@pytest.mark.parametrize("n", [284, 4352])
def test_grouped_product_matches_decoded_rows(n):
    """The grouped product against the decoded rows (decode_rotated, another kernel) times the input in fp64, for
    short rows and for rows whose column blocks outnumber the CTA's warps."""
    from lookatmyquant_b200 import artifact as A
    prod = _random_product(96, n, [1, 2, 3, 4], 21)
    tensors = {}
    for g, codes, rows, scales, table in prod.groups:
        tensors.update({g["key"] + ".codes": codes, g["key"] + ".rows": rows, g["key"] + ".scales": scales,
                        g["key"] + ".table": table})
    Wd = A.decode_rotated(tensors, prod.meta).double()
    xr = torch.randn(5, n, generator=torch.Generator().manual_seed(n)).float().cuda()
    y = A.product_rotated([prod], xr)[0].double()
    ref = xr.double() @ Wd.T
    assert (y - ref).abs().max() <= 1e-5 * ref.abs().max()
