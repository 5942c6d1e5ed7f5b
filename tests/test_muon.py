"""Muon: CPU parity with the unmodified reference optimizer, and the tcgen05
Newton-Schulz path vs the fp32 iteration on GPU."""
import pytest
import torch

import ref_oracle


def _params(seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(64, 48, generator=g), torch.randn(32, 96, generator=g), torch.randn(48, generator=g)]


@pytest.mark.skipif(not ref_oracle.available(), reason="reference not installed under baseline/_ref")
def test_muon_matches_reference_on_cpu():
    """Muon group: optimizer steps match the reference Muon.  Adam group: the update
    function matches (the reference's Muon cannot build an Adam group: its key check
    rejects both with and without ``use_adam``)."""
    from tinytron_b200.optim import Muon
    from tinytron_b200.optim.muon import adam_update

    with ref_oracle.cpu_reference():
        from tinytron.optim.muon import Muon as RefMuon
        from tinytron.optim.muon import adam_update as ref_adam_update
    ours = [torch.nn.Parameter(p.clone()) for p in _params(0)[:2]]
    ref = [torch.nn.Parameter(p.clone()) for p in _params(0)[:2]]
    opt_o = Muon([{"params": ours, "use_muon": True, "lr": 0.02, "momentum": 0.95, "weight_decay": 0.1}])
    opt_r = RefMuon([{"params": ref, "use_muon": True, "lr": 0.02, "momentum": 0.95, "weight_decay": 0.1}])
    g = torch.Generator().manual_seed(1)
    for _ in range(3):
        grads = [torch.randn(p.shape, generator=g) for p in ours]
        for p, q, gr in zip(ours, ref, grads):
            p.grad = gr.clone()
            q.grad = gr.clone()
        opt_o.step()
        opt_r.step()
    for p, q in zip(ours, ref):
        assert torch.allclose(p, q, atol=1e-5, rtol=1e-5), (p - q).abs().max()
    gr = torch.randn(48, generator=g)
    b1o, b2o, b1r, b2r = (torch.zeros(48) for _ in range(4))
    for step in (1, 2):
        uo = adam_update(gr.clone(), b1o, b2o, step, (0.9, 0.95), 1e-10)
        ur = ref_adam_update(gr.clone(), b1r, b2r, step, (0.9, 0.95), 1e-10)
        assert torch.allclose(uo, ur)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(256, 2048), (2048, 2048), (1024, 384), (5504, 2048)])
def test_newton_schulz_tcgen05_matches_fp32(shape):
    from tinytron_b200.optim.muon import NS_COEFFS, zeropower_via_newtonschulz5

    g = torch.Generator(device="cuda").manual_seed(0)
    G = torch.randn(*shape, device="cuda", generator=g)
    out = zeropower_via_newtonschulz5(G, 5)
    a, b, c = NS_COEFFS
    X = G.double()
    if X.size(0) > X.size(1):
        X = X.mT
    X = X / (X.norm() + 1e-7)
    for _ in range(5):
        A = X @ X.mT
        X = a * X + (b * A + c * A @ A) @ X
    if G.size(0) > G.size(1):
        X = X.mT
    err = ((out.double() - X).norm() / X.norm()).item()
    assert out.shape == G.shape and err < 3e-2, err
