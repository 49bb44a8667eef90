"""The KL probe head (compiler.py:176-187) against a plain PyTorch fp32 restatement of the reference's arithmetic:
bf16 logits from an fp32 accumulation, log_softmax in fp32, KL = Σ_t w_t Σ_v exp(lr)(lr − lp) / Σ_t w_t. Tolerance:
1e-4 nats on the mean KL (the bar for the KL probe), 1e-3 relative per position."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def torch_kl(h, h_ref, E, w=None):
    """The reference's formula, in fp64 on the device from fp32 logits rounded to bf16 (the model's lm_head output)."""
    def logp(x):
        z = (x.double() @ E.double().T).float().to(torch.bfloat16).float()
        return torch.log_softmax(z.double(), -1)
    lr, lp = logp(h_ref), logp(h)
    kl = (lr.exp() * (lr - lp)).sum(-1)
    w = torch.ones(len(kl), dtype=torch.float64, device=kl.device) if w is None else w.double()
    return float((kl * w).sum() / w.sum()), kl, lr


@pytest.mark.parametrize("ntok,d,V", [(300, 96, 1000), (1024, 960, 4096 + 37), (129, 64, 256)])
def test_kl_matches_torch(ntok, d, V):
    from lookatmyquant_b200.kl import KLReference
    g = torch.Generator(device="cuda").manual_seed(ntok + d + V)
    E = (0.5 * torch.randn(V, d, device="cuda", generator=g)).to(torch.bfloat16)
    h_ref = torch.randn(ntok, d, device="cuda", generator=g).to(torch.bfloat16)
    h = (h_ref.float() + 0.05 * torch.randn(ntok, d, device="cuda", generator=g)).to(torch.bfloat16)
    w = 1.0 + (torch.rand(ntok, device="cuda", generator=g) < 0.2).float() * 2.0
    ref = KLReference(h_ref, E)
    value, per_pos = ref.kl(h, w, per_position=True)
    want, kl_t, lr = torch_kl(h, h_ref, E, w)
    assert abs(value - want) <= 1e-4
    assert (per_pos.double() - kl_t).abs().max() <= 1e-3 * kl_t.abs().max() + 1e-5
    # the stored reference distribution: equal to fp32 precision except where the kernel's fp32 accumulation and
    # torch's round a logit to different bf16 neighbours (a bf16 step at |z| ~ 16 is 0.125)
    pr = lr.exp()
    close = (ref.p[:, :V].double() - pr).abs() <= 1e-5 * pr + 1e-12  # lse_ref is fp32: an ulp at |lse| ~ 30 is 2e-6
    assert close.double().mean() >= 0.999
    assert (ref.P - 1.0).abs().max() <= 1e-4


def test_kl_floor_is_exactly_zero():
    """The unquantized model probed against itself: the same passes, the same partial order — zero, as the
    reference's floor (lp == lr) is."""
    from lookatmyquant_b200.kl import KLReference
    g = torch.Generator(device="cuda").manual_seed(1)
    E = (0.5 * torch.randn(2000, 128, device="cuda", generator=g)).to(torch.bfloat16)
    h = torch.randn(500, 128, device="cuda", generator=g).to(torch.bfloat16)
    ref = KLReference(h, E)
    value, per_pos = ref.kl(h, per_position=True)
    assert value == 0.0 and bool((per_pos == 0).all())


def test_kl_matches_reference_evaluate(golden):
    """quantize.evaluate (quantize.py:903-920; the formula of compiler.py:180-187) of a tiny random-init bf16 Llama
    against a copy with one piece perturbed, run by the reference in make_golden.py: the KL head kernel on the two
    models' recorded final hidden states and the tied lm_head gives the same mean KL to 1e-4 nats."""
    from lookatmyquant_b200.kl import KLReference
    g = golden("kl")
    bf = lambda a: torch.as_tensor(a).view(torch.bfloat16).cuda()
    ref = KLReference(bf(g["h_ref"]), bf(g["E"]))
    value, per_pos = ref.kl(bf(g["h_probe"]), per_position=True)
    assert abs(value - float(g["kl"])) <= 1e-4
    assert (per_pos.cpu().double() - torch.as_tensor(g["kl_pos"]).double()).abs().max() <= 1e-3
    assert ref.kl(bf(g["h_ref"])) == 0.0
