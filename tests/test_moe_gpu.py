"""MoE device kernels (routing, layout, row movement, grouped tcgen05 GEMMs) against
plain fp32 PyTorch computations of the same ops."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def ext():
    from tinytron_b200.ops import _ext

    return _ext.load()


def rel_err(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _route(N, E, k, seed=0, skew=0.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    logits = torch.randn(N, E, device="cuda", generator=g)
    logits[:, 0] += skew  # uneven expert loads
    w = torch.empty(N, k, device="cuda")
    sel = torch.empty(N, k, device="cuda", dtype=torch.int32)
    ext().moe_topk_softmax(logits, k, w, sel)
    return logits, w, sel


def _layout(sel, E, align=128):
    C = ext()
    P = sel.numel()
    cap = C.moe_row_capacity(P, E, align)
    grp_off = torch.empty(E + 1, device="cuda", dtype=torch.int32)
    slot = torch.empty(P, device="cuda", dtype=torch.int32)
    row_pair = torch.empty(cap, device="cuda", dtype=torch.int32)
    C.moe_layout(sel.reshape(-1), E, grp_off, slot, row_pair, align)
    return cap, grp_off, slot, row_pair


@pytest.mark.parametrize("E,k", [(64, 8), (8, 2), (256, 1)])
def test_topk_softmax_matches_torch(E, k):
    logits, w, sel = _route(1000, E, k)
    tv, ti = torch.topk(logits, k, dim=-1)
    assert torch.equal(sel.long(), ti)
    assert torch.allclose(w, torch.softmax(tv, -1), atol=1e-6)
    # backward
    dw = torch.randn_like(w)
    dl = torch.empty_like(logits)
    ext().moe_topk_softmax_bwd(dw, w, sel, dl)
    lg = logits.clone().requires_grad_(True)
    tv2 = torch.gather(lg, 1, ti)
    torch.softmax(tv2, -1).backward(dw)
    assert torch.allclose(dl, lg.grad, atol=1e-6)


@pytest.mark.parametrize("N,E,k,align", [(3000, 16, 4, 128), (1000, 16, 4, 128), (40000, 64, 8, 256),
                                         (20000, 256, 2, 1), (9000, 64, 8, 128), (24, 64, 8, 1)])
def test_layout_segments_are_aligned_stable_and_complete(N, E, k, align):
    # pair counts <= 8192 take the one-launch kernel, larger ones the count/scan/place kernels
    _, _, sel = _route(N, E, k, skew=2.0)
    cap, grp_off, slot, row_pair = _layout(sel, E, align)
    off = grp_off.cpu().tolist()
    counts = torch.bincount(sel.reshape(-1).long(), minlength=E).cpu().tolist()
    flat = sel.reshape(-1).cpu()
    sl = slot.cpu()
    rp = row_pair.cpu()
    assert off[0] == 0 and off[-1] <= cap
    for e in range(E):
        assert off[e] % align == 0
        assert off[e + 1] - off[e] == (counts[e] + align - 1) // align * align
        pairs = torch.nonzero(flat == e).squeeze(-1)
        assert torch.equal(sl[pairs], torch.arange(off[e], off[e] + counts[e], dtype=torch.int32))  # stable
        assert torch.equal(rp[off[e]:off[e] + counts[e]].long(), pairs)
        assert (rp[off[e] + counts[e]:off[e + 1]] == -1).all()
    assert ext().status_read(0) == 0


@pytest.mark.parametrize("N,lo", [(32, 8), (3000, 24)])
def test_layout_remap_matches_precomputed_local_ids(N, lo):
    """remap_lo: ids in [lo, lo + E_l) become local experts, all others the last group."""
    C = ext()
    E, k, E_l = 64, 8, 8
    _, _, sel = _route(N, E, k)
    flat = sel.reshape(-1)
    local = flat - lo
    local = torch.where((local >= 0) & (local < E_l), local, torch.full_like(local, E_l)).contiguous()
    outs = []
    for ids, remap in ((local, -1), (flat.contiguous(), lo)):
        P = ids.numel()
        cap = C.moe_row_capacity(P, E_l + 1, 1)
        grp = torch.empty(E_l + 2, device="cuda", dtype=torch.int32)
        slot = torch.empty(P, device="cuda", dtype=torch.int32)
        rp = torch.empty(cap, device="cuda", dtype=torch.int32)
        C.moe_layout(ids, E_l + 1, grp, slot, rp, 1, remap)
        outs.append((grp, slot, rp[:int(grp[-1])]))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    assert ext().status_read(0) == 0


def test_gather_combine_and_backward():
    C = ext()
    N, E, k, H = 777, 8, 2, 256
    _, w, sel = _route(N, E, k)
    cap, grp_off, slot, row_pair = _layout(sel, E)
    x = torch.randn(N, H, device="cuda").bfloat16()
    xr = torch.full((cap, H), float("nan"), device="cuda", dtype=torch.bfloat16)
    C.moe_gather_rows(x, row_pair, grp_off, k, xr)
    total = int(grp_off[-1])
    rp = row_pair[:total].long()
    ref = torch.where((rp >= 0)[:, None], x[(rp.clamp(min=0) // k)], torch.zeros_like(x[:1]))
    assert torch.equal(xr[:total], ref)
    y_rows = torch.randn(cap, H, device="cuda").bfloat16()
    out = torch.empty(N, H, device="cuda", dtype=torch.bfloat16)
    C.moe_combine(y_rows, slot, w, k, out)
    gathered = y_rows[slot.long()].float().view(N, k, H)
    ref = (gathered * w[..., None]).sum(1)
    assert rel_err(out, ref) < 5e-3
    dout = torch.randn(N, H, device="cuda").bfloat16()
    dy = torch.full((cap, H), float("nan"), device="cuda", dtype=torch.bfloat16)
    dw = torch.empty_like(w)
    C.moe_combine_bwd(dout, y_rows, row_pair, w, grp_off, k, dy, dw)
    ref_dw = (gathered * dout.float()[:, None, :]).sum(-1)
    assert rel_err(dw, ref_dw) < 1e-4
    ref_dy = torch.zeros(total, H, device="cuda")
    valid = rp >= 0
    ref_dy[valid] = w.reshape(-1)[rp[valid]][:, None] * dout.float()[rp[valid] // k]
    assert rel_err(dy[:total], ref_dy) < 5e-3
    assert not torch.isnan(dy[:total].float()).any()


def _expert_setup(N=1500, E=8, k=2, H=256, I=384, seed=0, align=128):
    g = torch.Generator(device="cuda").manual_seed(seed)
    _, w, sel = _route(N, E, k, seed=seed, skew=1.5)
    cap, grp_off, slot, row_pair = _layout(sel, E, align)
    x = (torch.randn(N, H, device="cuda", generator=g)).bfloat16()
    wg = (torch.randn(E, I, H, device="cuda", generator=g) * 0.05).bfloat16()
    wu = (torch.randn(E, I, H, device="cuda", generator=g) * 0.05).bfloat16()
    wd = (torch.randn(E, H, I, device="cuda", generator=g) * 0.05).bfloat16()
    xr = torch.empty(cap, H, device="cuda", dtype=torch.bfloat16)
    ext().moe_gather_rows(x, row_pair, grp_off, k, xr)
    return dict(N=N, E=E, k=k, H=H, I=I, w=w, sel=sel, cap=cap, grp_off=grp_off, slot=slot, row_pair=row_pair,
                x=x, wg=wg, wu=wu, wd=wd, xr=xr)


def _segments(s):
    off = s["grp_off"].cpu().tolist()
    return [(e, off[e], off[e + 1]) for e in range(s["E"])]


# (segment alignment, CTA-pair kernel): 256-aligned segments run on the pair kernel
LAYOUTS = [(128, False), (256, True)]


@pytest.mark.parametrize("align,pair", LAYOUTS)
def test_grouped_swiglu_down_forward(align, pair):
    C = ext()
    s = _expert_setup(align=align)
    cap, E, H, I = s["cap"], s["E"], s["H"], s["I"]
    w_gu = torch.cat([s["wg"].reshape(E * I, H), s["wu"].reshape(E * I, H)], 0)
    act = torch.empty(cap, I, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(cap, 2 * I, device="cuda", dtype=torch.bfloat16)
    C.moe_gemm_swiglu(s["xr"], w_gu, act, gu, s["grp_off"], E, pair)
    y = torch.empty(cap, H, device="cuda", dtype=torch.bfloat16)
    C.moe_gemm(act, s["wd"].reshape(E * H, I), y, s["grp_off"], E, False, H, 0, 0, pair)
    for e, a, b in _segments(s):
        if b == a:
            continue
        xe = s["xr"][a:b].float()
        g_ = xe @ s["wg"][e].float().t()
        u_ = xe @ s["wu"][e].float().t()
        act_ref = torch.nn.functional.silu(g_) * u_
        assert rel_err(gu[a:b, :I], g_) < 1e-2 and rel_err(gu[a:b, I:], u_) < 1e-2
        assert rel_err(act[a:b], act_ref) < 1e-2, e
        assert rel_err(y[a:b], act[a:b].float() @ s["wd"][e].float().t()) < 1e-2, e


@pytest.mark.parametrize("align,pair", LAYOUTS)
def test_grouped_backward_gemms(align, pair):
    C = ext()
    s = _expert_setup(seed=1, align=align)
    cap, E, H, I = s["cap"], s["E"], s["H"], s["I"]
    gen = torch.Generator(device="cuda").manual_seed(7)
    gu = (torch.randn(cap, 2 * I, device="cuda", generator=gen)).bfloat16()
    dy = (torch.randn(cap, H, device="cuda", generator=gen)).bfloat16()
    total = int(s["grp_off"][-1])
    pad = s["row_pair"][:total] < 0
    dy[:total][pad] = 0  # pad rows carry no gradient
    act = (torch.randn(cap, I, device="cuda", generator=gen)).bfloat16()
    act[:total][pad] = 0
    # down dgrad fused with the SwiGLU backward
    dgu = torch.empty(cap, 2 * I, device="cuda", dtype=torch.bfloat16)
    C.moe_gemm_dswiglu(dy, s["wd"].reshape(E * H, I), gu, dgu, s["grp_off"], E, pair)
    # gate|up dgrad (B = stacked gate / up weights, MN-major, split at I)
    w_gu = torch.cat([s["wg"].reshape(E * I, H), s["wu"].reshape(E * I, H)], 0)
    dx = torch.empty(cap, H, device="cuda", dtype=torch.bfloat16)
    C.moe_gemm(dgu, w_gu, dx, s["grp_off"], E, True, I, I, E * I, pair)
    # weight grads, accumulated into fp32
    gwd = torch.ones(E * H, I, device="cuda")
    C.moe_gemm_wgrad(dy, act, gwd, s["grp_off"], E, True, pair)
    gwg = torch.empty(E * I, H, device="cuda")
    C.moe_gemm_wgrad(dgu[:, :I], s["xr"], gwg, s["grp_off"], E, False, pair)
    for e, a, b in _segments(s):
        wd_e = s["wd"][e].float()
        if b == a:
            assert torch.all(gwd[e * H:(e + 1) * H] == 1) and torch.all(gwg[e * I:(e + 1) * I] == 0)
            continue
        dact = dy[a:b].float() @ wd_e
        g_, u_ = gu[a:b, :I].float(), gu[a:b, I:].float()
        sg = torch.sigmoid(g_)
        dg = dact * u_ * sg * (1 + g_ * (1 - sg))
        du = dact * g_ * sg
        assert rel_err(dgu[a:b, :I], dg) < 1e-2 and rel_err(dgu[a:b, I:], du) < 1e-2, e
        dx_ref = dgu[a:b, :I].float() @ s["wg"][e].float() + dgu[a:b, I:].float() @ s["wu"][e].float()
        assert rel_err(dx[a:b], dx_ref) < 1e-2, e
        assert rel_err(gwd[e * H:(e + 1) * H] - 1, dy[a:b].float().t() @ act[a:b].float()) < 1e-3, e
        assert rel_err(gwg[e * I:(e + 1) * I], dgu[a:b, :I].float().t() @ s["xr"][a:b].float()) < 1e-3, e
    assert ext().status_read(0) == 0


def test_moe_module_forward_backward_matches_fp32_with_same_routing():
    """The MoE block on the device path vs an fp32 CPU restatement that uses the same
    expert selection (bf16 router logits can order near-ties differently from fp32)."""
    from tinytron_b200.models import ModelConfig
    from tinytron_b200.models.modules.mlp import MoE
    from tinytron_b200 import ops

    cfg = ModelConfig(block_size=256, vocab_size=128, num_layer=1, num_attention_heads=2, num_key_value_heads=1,
                      hidden_size=256, intermediate_size=512, use_moe=True, num_experts=8, num_experts_per_tok=2,
                      moe_intermediate_size=384, init_std=0.05, seed=4)
    m = MoE(cfg, 0, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(2, 200, 256, device="cuda", generator=g).bfloat16().requires_grad_(True)
    gy = torch.randn(2, 200, 256, device="cuda", generator=g)
    y, logits = m(x)
    (y.float() * gy).sum().backward()
    _, sel = torch.topk(logits.detach().float().view(-1, 8), 2, dim=-1)

    params = {n: p.detach().float().cpu().requires_grad_(True) for n, p in m.named_parameters()}
    xf = x.detach().float().cpu().requires_grad_(True)
    lg = xf.view(-1, 256) @ params["router.weight"].t()
    w_ref = torch.softmax(torch.gather(lg, 1, sel.cpu()), -1)
    y_ref = ops.moe_experts(xf.view(-1, 256), sel.cpu(), w_ref, params["experts_gate_weights"],
                            params["experts_up_weights"], params["experts_down_weights"])
    (y_ref * gy.view(-1, 256).cpu()).sum().backward()
    assert rel_err(y.view(-1, 256).cpu(), y_ref) < 2e-2
    assert rel_err(x.grad.cpu(), xf.grad) < 3e-2
    for n, p in m.named_parameters():
        assert rel_err(p.grad.cpu(), params[n].grad) < 3e-2, n
    assert ext().status_read(0) == 0
