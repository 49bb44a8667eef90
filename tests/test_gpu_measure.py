"""The measure sweep's pieces (compiler.py:134-291) on a two-layer model of the SmolLM2 architecture: H from the
calibration pass against the reference's fp32 Xᵀ·X / n of the same activations, the KL floor, and one probe."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_capture_matches_fp32_statistics():
    from lookatmyquant_b200 import measure
    model = measure.build_model(layers=2)
    chunks = [measure.zipf_tokens(2, 96, model.config.vocab_size, 3).cuda()]
    H = measure.capture(model, [0], chunks)
    xs = []
    h = model.model.layers[0].mlp.down_proj.register_forward_pre_hook(lambda m, a: xs.append(a[0].reshape(-1, a[0].shape[-1])))
    with torch.no_grad():
        model.model(chunks[0], use_cache=False)
    h.remove()
    x = xs[0].float()
    ref = (x.T @ x / len(x)).double()
    got = H[(0, "mlp.down_proj")]
    assert (got - ref).norm() <= 1e-5 * ref.norm()
    assert set(H) == {(0, "self_attn.q_proj"), (0, "self_attn.o_proj"), (0, "mlp.gate_proj"), (0, "mlp.down_proj")}


def test_probe_floor_and_one_option():
    from lookatmyquant_b200 import measure
    res = measure.run(layers=range(1), options=("tr2",), n_layers=2, windows=2, T=128, calib=2, chunk=2, log=lambda s: None)
    assert res["kl floor"] == 0.0
    assert res["probes"] == 7
    dkl = [r["dkl"] for r in res["records"]]
    assert all(d >= -1e-6 for d in dkl) and max(dkl) > 0


def test_probe_from_a_cached_layer_input_equals_the_full_forward():
    """The hidden states of a probe that starts at the quantized piece's layer (earlier layers' outputs kept from the
    reference pass) are bit-identical to a full forward of the modified model."""
    from lookatmyquant_b200 import measure
    model = measure.build_model(layers=3)
    held = measure.zipf_tokens(4, 64, model.config.vocab_size, 5)
    probe = measure.Probe(model, held, batch=2)
    assert probe.kl(start=0) == 0.0 and probe.kl(start=2) == 0.0
    mod = model.model.layers[1].mlp.up_proj
    orig = mod.weight.data.clone()
    mod.weight.data = (orig.float() * 1.01).to(torch.bfloat16)
    assert torch.equal(probe.hidden(start=1), probe.hidden())
    assert probe.kl(start=1) == probe.kl() and probe.kl() > 0
    mod.weight.data = orig


def test_sweep_split_by_piece_equals_the_whole_sweep():
    """Two ranks' shares of the sweep (run one after the other on this GPU, each with its own model replica) hold
    every piece once, and each record's KL equals the single-rank sweep's exactly."""
    from lookatmyquant_b200 import measure
    kw = dict(layers=range(2), options=("tr2",), n_layers=2, windows=2, T=128, calib=2, chunk=2, log=lambda s: None)
    whole = measure.run(**kw)
    parts = [measure.run(**kw, rank=r, world=2) for r in range(2)]
    assert sum(p["probes"] for p in parts) == whole["probes"] == 14
    got = {(r["item"], r["option"]): r["dkl"] for p in parts for r in p["records"]}
    want = {(r["item"], r["option"]): r["dkl"] for r in whole["records"]}
    assert got == want
    assert {r["item"] for r in parts[0]["records"]}.isdisjoint({r["item"] for r in parts[1]["records"]})


def test_trellis_linear_matches_the_dense_word():
    """The probe's quantized piece as a TrellisLinear (rotations through the factors, the tensor-core GEMM from the
    int16 states) against x·Wᵀ with the dense word W = word.matrix(), within the bf16-operand bar (1e-2)."""
    from lookatmyquant_b200 import codes
    from lookatmyquant_b200.artifact import TrellisLinear
    g = torch.Generator().manual_seed(3)
    W = (0.02 * torch.randn(640, 960, generator=g, dtype=torch.float64)).cuda()
    A = torch.randn(4096, 960, generator=g, dtype=torch.float64).cuda()
    H = A.T @ A / 4096
    word = codes.ldlq_words([W], H, codes.TrellisCode(12, 2, T=320), [7])[0]
    x = torch.randn(2, 700, 960, generator=g).to(torch.bfloat16).cuda()
    y = TrellisLinear(word)(x)
    assert y.shape == (2, 700, 640) and y.dtype == torch.bfloat16
    ref = x.double().reshape(-1, 960) @ word.matrix().T
    assert (y.reshape(-1, 640).double() - ref).abs().max() <= 1e-2 * ref.abs().max()


def test_trellis_linear_launches_no_library_gemm():
    """The quantized piece's forward runs this library's kernels and torch's elementwise casts only: no cuBLAS or
    other library GEMM."""
    from torch.profiler import ProfilerActivity, profile
    from lookatmyquant_b200 import codes
    from lookatmyquant_b200.artifact import TrellisLinear
    g = torch.Generator().manual_seed(4)
    W = (0.02 * torch.randn(320, 960, generator=g, dtype=torch.float64)).cuda()
    word = codes.ldlq_words([W], None, codes.TrellisCode(12, 3, T=320), [9])[0]
    lin = TrellisLinear(word)
    x = torch.randn(1024, 960, generator=g).to(torch.bfloat16).cuda()
    lin(x)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        lin(x)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    assert any("trellis_gemm_kernel" in nm for nm in names)
    assert any("rht_rows" in nm for nm in names)
    library = [nm for nm in names if ("gemm" in nm.lower() or "cutlass" in nm.lower() or "xmma" in nm.lower())
               and "lamq" not in nm]
    assert not library, library


def test_probe_kl_through_trellis_linear_matches_the_dense_piece():
    """The sweep with each quantized piece as a TrellisLinear gives every record's KL within 1e-4 nats of the sweep
    that writes the dense bf16 word into the model (the reference's way)."""
    from lookatmyquant_b200 import measure
    kw = dict(layers=range(2), options=("tr2", "tr4"), n_layers=2, windows=2, T=256, calib=2, chunk=2,
              log=lambda s: None)
    fused = measure.run(**kw)
    dense = measure.run(**kw, dense_piece=True)
    a = {(r["item"], r["option"]): r["dkl"] for r in fused["records"]}
    b = {(r["item"], r["option"]): r["dkl"] for r in dense["records"]}
    assert a.keys() == b.keys() and len(a) == 28
    assert max(abs(a[k] - b[k]) for k in a) <= 1e-4
    assert max(b.values()) > 1e-4  # the pieces do move the KL
