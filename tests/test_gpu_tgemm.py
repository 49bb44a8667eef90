"""The trellis-dequant GEMM (lamq_trellis_gemm): weights decoded from trellis states into the tensor cores' shared
memory operand, fp32 accumulation. Checked against the same product formed in fp64 from the bf16-rounded table
values (y = S·Σ bf16(V[state])·bf16(x)) — only the fp32 summation order differs: 1e-5 of the largest output — and
against the config-5 bar (dense bf16 product of the decoded weights, 1e-2 relative)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _path(rows, n, k, seed):
    """Random trellis paths from state 0 (int64 rows x n)."""
    g = np.random.default_rng(seed)
    sym = g.integers(0, 1 << k, size=(rows, n))
    st = np.zeros((rows, n), dtype=np.int64)
    s = np.zeros(rows, dtype=np.int64)
    for j in range(n):
        s = ((s << k) | sym[:, j]) & 4095
        st[:, j] = s
    return st


def _groups(m, n, widths, seed, states_source=False):
    """Row groups of an m-row matrix (rows permuted among the groups), each with packed codes or int16 states."""
    from lookatmyquant_b200 import artifact as A
    gen = torch.Generator().manual_seed(seed)
    perm = torch.randperm(m, generator=gen)
    cuts = np.linspace(0, m, len(widths) + 1).astype(int)
    out = []
    for i, k in enumerate(widths):
        rows = perm[cuts[i]:cuts[i + 1]].sort().values.to(torch.int32).cuda()
        st = torch.as_tensor(_path(rows.numel(), n, k, seed + i)).cuda()
        out.append({"k": k, "rows": rows, "states": st.to(torch.int16).contiguous(),
                    "codes": None if states_source else A.pack_trellis(st, k),
                    "scales": (0.5 + torch.rand(rows.numel(), generator=gen)).float().cuda(),
                    "table": torch.randn(4096, generator=gen).float().cuda()})
    return out


def _run(groups, n, x, m, y_bf16=False):
    from lookatmyquant_b200 import _lib, artifact as A
    from lookatmyquant_b200._lib import ptr
    y = torch.full((x.shape[0], m), float("nan"), device="cuda",
                   dtype=torch.bfloat16 if y_bf16 else torch.float32)
    descs = [_lib.GemmGroup(ptr(g["codes"]), None if g["codes"] is not None else ptr(g["states"]),
                            g["states"].stride(0), g["rows"].numel(), g["k"], 12, ptr(g["scales"]), ptr(g["table"]),
                            ptr(g["rows"]), ptr(y), y.stride(0), ptr(x), x.stride(0), n, 0) for g in groups]
    status = A.gemm_groups(descs, x.shape[0], x.device, y_bf16)
    assert int(status.item()) == 0
    return y


def _reference(groups, x, m):
    ref = torch.zeros(x.shape[0], m, dtype=torch.float64, device="cuda")
    xd = x.double()
    for g in groups:
        W = g["table"].to(torch.bfloat16).double()[g["states"].long()] * g["scales"].double()[:, None]
        ref[:, g["rows"].long()] = xd @ W.T
    return ref


@pytest.mark.parametrize("n,nvec", [(200, 64), (2560, 100), (960, 256), (4352, 300), (2560, 600), (320, 2048)])
@pytest.mark.parametrize("source", ["packed", "states"])
def test_gemm_matches_fp64_of_the_bf16_operands(n, nvec, source):
    """Mixed widths in one launch (k = 1..4, rows permuted), ragged n (a last slice of 8 or 32 columns), vector
    counts below, at and between the accumulator widths (one accumulator, two, a ragged last block)."""
    m = 300
    groups = _groups(m, n, [1, 2, 3, 4, 2], 7 * n + nvec, states_source=(source == "states" and n % 8 == 0))
    x = torch.randn(nvec, n, generator=torch.Generator().manual_seed(nvec)).to(torch.bfloat16).cuda()
    y = _run(groups, n, x, m)
    ref = _reference(groups, x, m)
    assert not torch.isnan(y).any()
    assert (y.double() - ref).abs().max() <= 1e-5 * ref.abs().max()


def test_gemm_bf16_output_and_strided_input():
    from lookatmyquant_b200 import artifact as A
    m, n = 256, 1024
    groups = _groups(m, n, [2, 3], 5)
    base = torch.randn(130, n + 8, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).cuda()
    x = base[:, 8:]  # rows 16-byte aligned at a leading dimension of n + 8
    y = _run(groups, n, x, m, y_bf16=True)
    ref = _reference(groups, x, m)
    assert y.dtype == torch.bfloat16
    assert (y.double() - ref).abs().max() <= 1e-2 * ref.abs().max()
    assert torch.equal(y, _run(groups, n, x, m).to(torch.bfloat16))  # the same fp32 sums, rounded once
    assert A._bf16_operand(x, x.device).data_ptr() == x.data_ptr()


def test_gemm_is_deterministic_and_many_groups():
    """More than 16 groups take several launches; repeated calls give identical bits."""
    m, n = 2000, 512
    groups = _groups(m, n, [1, 2, 3, 4] * 5, 9)
    x = torch.randn(512, n, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).cuda()
    y1, y2 = _run(groups, n, x, m), _run(groups, n, x, m)
    assert torch.equal(y1, y2)
    ref = _reference(groups, x, m)
    assert (y1.double() - ref).abs().max() <= 1e-5 * ref.abs().max()


def test_layer_in_one_launch_equals_stage_by_stage():
    """Groups over different inputs (a layer's stages: three inputs of 2560, 4096 and 9728 columns, 17 groups, so
    two launches) give every output exactly what each stage's own launch gives."""
    from lookatmyquant_b200 import _lib, artifact as A
    from lookatmyquant_b200._lib import ptr
    nvec = 300
    specs = [(640, 2560, [1, 2, 3, 4, 2, 3]), (384, 4096, [2, 3, 4, 1, 2]), (300, 9728, [3, 1, 4, 2, 2, 3])]
    stages = []
    for m, n, widths in specs:
        groups = _groups(m, n, widths, m + n)
        x = torch.randn(nvec, n, generator=torch.Generator().manual_seed(n)).to(torch.bfloat16).cuda()
        stages.append((m, n, groups, x))
    alone = [_run(groups, n, x, m) for m, n, groups, x in stages]
    ys = [torch.full((nvec, m), float("nan"), device="cuda") for m, _, _, _ in stages]
    descs = [_lib.GemmGroup(ptr(g["codes"]), None, 0, g["rows"].numel(), g["k"], 12, ptr(g["scales"]),
                            ptr(g["table"]), ptr(g["rows"]), ptr(y), y.stride(0), ptr(x), x.stride(0), n, 0)
             for (m, n, groups, x), y in zip(stages, ys) for g in groups]
    assert len(descs) == 17
    st = A.gemm_groups(descs, nvec, torch.device("cuda"))
    assert int(st.item()) == 0
    for y, ref in zip(ys, alone):
        assert torch.equal(y, ref)


def test_trellis_product_uses_the_gemm_from_64_vectors(golden):
    """TrellisProduct on the reference's packed entry (artifact.npz): from 64 vectors the tensor-core GEMM, within
    the config-5 bar of the fp64 product of the reference's decoded weights."""
    from lookatmyquant_b200 import _lib, artifact as A
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
    prod = A.TrellisProduct(tensors, A.grouped_matrix_meta("w", [200, 200], groups))
    x = torch.randn(2048, 200, dtype=torch.float64, generator=torch.Generator().manual_seed(3)).cuda()
    before = _lib.load().lamq_kernel_launches()
    y = prod(x).double().cpu().numpy()
    assert _lib.load().lamq_kernel_launches() > before
    xr = Rotation.from_signs(torch.as_tensor(g["signs"]).double()).rows(x).cpu().numpy()
    ref = xr @ g["decoded"].astype(np.float64).T
    assert np.abs(y - ref).max() <= 1e-2 * np.abs(ref).max()


@pytest.mark.parametrize("nvec", [513, 1000, 2048])
def test_decode_once_mode_equals_the_fused_decode(nvec):
    """From 513 vectors the weights are decoded once into the workspace and fed by TMA: the same products as the
    fused decode of the same groups, block of 512 vectors by block, bit for bit (packed and int16 sources, ragged n)."""
    m, n = 700, 2504
    for states_source in (False, True):
        groups = _groups(m, n, [4, 1, 3, 2], 3 * nvec, states_source=states_source)
        x = torch.randn(nvec, n, generator=torch.Generator().manual_seed(nvec)).to(torch.bfloat16).cuda()
        y = _run(groups, n, x, m)
        parts = [_run(groups, n, x[v:v + 512], m) for v in range(0, nvec, 512)]
        assert torch.equal(y, torch.cat(parts))
        ref = _reference(groups, x, m)
        assert (y.double() - ref).abs().max() <= 1e-5 * ref.abs().max()
