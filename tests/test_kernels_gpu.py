"""sm_100a kernels vs plain PyTorch fp32 references of the same ops."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def ext():
    from tinytron_b200.ops import _ext

    return _ext.load()


def rel_err(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


@pytest.mark.parametrize("M,D", [(1, 256), (37, 768), (512, 2048), (64, 5120)])
@pytest.mark.parametrize("with_delta", [False, True])
def test_add_rmsnorm_fwd_bwd(M, D, with_delta):
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, D, device="cuda", generator=g)
    delta = torch.randn(M, D, device="cuda", generator=g).bfloat16() if with_delta else None
    w = torch.rand(D, device="cuda", generator=g) + 0.5
    eps = 1e-6
    x_out = torch.empty_like(x)
    h = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    rstd = torch.empty(M, device="cuda")
    ext().add_rmsnorm_fwd(x, delta, w, x_out, h, rstd, eps)
    xr = x + (delta.float() if with_delta else 0)
    ref = w * (xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + eps))
    assert rel_err(x_out, xr) < 1e-6
    assert rel_err(h, ref) < 1e-2
    # backward
    gh = torch.randn(M, D, device="cuda", generator=g).bfloat16()
    gres = torch.randn(M, D, device="cuda", generator=g)
    xx = xr.clone().requires_grad_(True)
    ww = w.clone().requires_grad_(True)
    y = ww * (xx * torch.rsqrt(xx.pow(2).mean(-1, keepdim=True) + eps))
    y.backward(gh.float())
    gx = torch.empty_like(x)
    gd = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    dw = torch.ones(D, device="cuda")
    scratch = torch.empty(ext().rmsnorm_bwd_scratch_numel(M, D), device="cuda")
    ext().rmsnorm_bwd(gh, x_out, rstd, w, gres, gx, gd, dw, True, scratch)
    assert rel_err(gx, xx.grad + gres) < 1e-4
    assert rel_err(gd, xx.grad + gres) < 1e-2
    assert rel_err(dw - 1.0, ww.grad) < 1e-4


def _rope_ref(x, pos, theta=10000.0):
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d))
    fr = pos.float()[:, None] * inv[None]
    emb = torch.cat([fr, fr], -1)
    cos, sin = emb.cos(), emb.sin()
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    rot = torch.cat([-x2, x1], -1)
    return x * cos[:, None] + rot * sin[:, None]


@pytest.mark.parametrize("d", [64, 128])
def test_rope(d):
    from tinytron_b200.ops.rope import rope_tables

    B, T, H, off = 2, 100, 6, 7
    x = torch.randn(B * T, H * d + 64, device="cuda").bfloat16()
    cos, sin = rope_tables(d, 10000.0, 512, torch.device("cuda"))
    y = x.clone()
    ext().rope_inplace(y, cos, sin, T, off, H, d, False)
    pos = (torch.arange(B * T, device="cuda") % T) + off
    ref = _rope_ref(x[:, : H * d].float().view(B * T, H, d), pos).view(B * T, H * d)
    assert rel_err(y[:, : H * d], ref) < 1e-2
    assert torch.equal(y[:, H * d:], x[:, H * d:])
    z = y.clone()
    ext().rope_inplace(z, cos, sin, T, off, H, d, True)
    assert rel_err(z[:, : H * d], x[:, : H * d]) < 2e-2


@pytest.mark.parametrize("M,V", [(7, 1000), (64, 50304), (33, 8192)])
def test_cross_entropy(M, V):
    logits = (torch.randn(M, V, device="cuda") * 3).bfloat16()
    tgt = torch.randint(0, V, (M,), device="cuda")
    tgt[::5] = -100
    loss = torch.empty(M, device="cuda")
    lse = torch.empty(M, device="cuda")
    lg = logits.clone()
    ext().cross_entropy_fwd(lg, tgt, loss, lse, -100, True)
    lf = logits.float().requires_grad_(True)
    ref = F.cross_entropy(lf, tgt, ignore_index=-100, reduction="none")
    ref.sum().backward()
    assert rel_err(loss, ref) < 1e-4
    assert rel_err(lse, torch.logsumexp(logits.float(), -1)) < 1e-5
    assert rel_err(lg, lf.grad) < 1e-2


def test_embedding():
    V, D, M = 100, 256, 300
    table = torch.randn(V, D, device="cuda")
    idx = torch.randint(0, V, (M,), device="cuda")
    out = torch.empty(M, D, device="cuda")
    ext().embedding_fwd(idx, table, out)
    assert torch.equal(out, table[idx])
    g = torch.randn(M, D, device="cuda")
    gt = torch.zeros(V, D, device="cuda")
    ext().embedding_bwd(idx, g, gt)
    ref = torch.zeros(V, D, device="cuda").index_add_(0, idx, g)
    assert rel_err(gt, ref) < 1e-5


def test_adamw_matches_torch():
    n = 10007
    p = torch.randn(n, device="cuda")
    grads = [torch.randn(n, device="cuda") for _ in range(3)]
    ref_p = p.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref_p], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    ours = p.clone()
    scale = torch.tensor([0.5], device="cuda")
    for step, gr in enumerate(grads, 1):
        ref_p.grad = gr * 0.5
        opt.step()
        ext().adamw_step(ours, gr.clone(), m, v, p16, 1e-2, 0.9, 0.95, 1e-8, 0.1, step, scale)
    assert rel_err(ours, ref_p.detach()) < 1e-5
    assert rel_err(p16, ours) < 1e-2


def test_sumsq_and_clip():
    x = torch.randn(1_000_003, device="cuda")
    out = torch.zeros(1, device="cuda")
    scratch = torch.empty(148 * 8 + 64, device="cuda")
    ext().sumsq(x, out, scratch, False)
    assert rel_err(out, (x.double() ** 2).sum().float()) < 1e-5
    nrm = torch.empty(1, device="cuda")
    coef = torch.empty(1, device="cuda")
    ext().clip_coef(out, nrm, coef, 1.0)
    assert abs(nrm.item() - x.norm().item()) / x.norm().item() < 1e-5
    assert abs(coef.item() - min(1.0, 1.0 / (x.norm().item() + 1e-6))) < 1e-6


def _attn_ref(q, k, v, causal, offset=0):
    # q [B, Hq, T, d], k/v [B, Hkv, Tk, d]
    Hq, Hkv = q.shape[1], k.shape[1]
    k = k.repeat_interleave(Hq // Hkv, 1)
    v = v.repeat_interleave(Hq // Hkv, 1)
    s = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    if causal:
        T, Tk = q.shape[2], k.shape[2]
        mask = torch.arange(Tk, device=q.device)[None, :] <= (torch.arange(T, device=q.device)[:, None] + offset)
        s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    return torch.softmax(s, -1) @ v.float(), lse


@pytest.mark.parametrize("B,T,Hq,Hkv,d", [(1, 128, 2, 1, 128), (2, 300, 4, 2, 128), (2, 1024, 16, 4, 128),
                                           (1, 200, 4, 4, 64), (1, 4096, 2, 1, 128)])
@pytest.mark.parametrize("causal", [True, False])
def test_attn_fwd_packed_qkv(B, T, Hq, Hkv, d, causal):
    W = (Hq + 2 * Hkv) * d
    qkv = (torch.randn(B * T, W, device="cuda")).bfloat16()
    o = torch.empty(B * T, Hq * d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, T, device="cuda")
    ext().attn_fwd(qkv, qkv, qkv, 0, Hq * d, (Hq + Hkv) * d, B, T, T, Hq, Hkv, d, o, lse, 1 / math.sqrt(d),
                   causal, 0)
    x = qkv.view(B, T, Hq + 2 * Hkv, d).transpose(1, 2)
    q, k, v = x[:, :Hq], x[:, Hq:Hq + Hkv], x[:, Hq + Hkv:]
    ref, ref_lse = _attn_ref(q, k, v, causal)
    got = o.view(B, T, Hq, d).transpose(1, 2)
    assert rel_err(got, ref) < 2e-2
    assert (lse - ref_lse).abs().max().item() < 2e-2
    assert ext().status_read(0) == 0


@pytest.mark.parametrize("B,T,Hq,Hkv,d", [(1, 128, 2, 1, 128), (2, 300, 4, 2, 128), (2, 1024, 16, 4, 128),
                                           (1, 200, 4, 4, 64), (1, 2048, 4, 1, 128)])
@pytest.mark.parametrize("causal", [True, False])
def test_attn_bwd_packed_qkv(B, T, Hq, Hkv, d, causal):
    W = (Hq + 2 * Hkv) * d
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = torch.randn(B * T, W, device="cuda", generator=g).bfloat16()
    o = torch.empty(B * T, Hq * d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, T, device="cuda")
    scale = 1 / math.sqrt(d)
    ext().attn_fwd(qkv, qkv, qkv, 0, Hq * d, (Hq + Hkv) * d, B, T, T, Hq, Hkv, d, o, lse, scale, causal, 0)
    do = torch.randn(B * T, Hq * d, device="cuda", generator=g).bfloat16()
    dqkv = torch.full((B * T, W), float("nan"), device="cuda", dtype=torch.bfloat16)
    dq_acc = torch.empty(B * T, Hq * d, device="cuda")
    delta = torch.empty(ext().attn_bwd_scratch_numel(B, Hq, T), device="cuda")
    ext().attn_bwd(qkv, qkv, qkv, o, do, 0, Hq * d, (Hq + Hkv) * d, lse, B, T, Hq, Hkv, d,
                   dqkv, 0, dqkv, Hq * d, dqkv, (Hq + Hkv) * d, dq_acc, delta, scale, causal)
    x = qkv.float().view(B, T, Hq + 2 * Hkv, d).transpose(1, 2).detach().requires_grad_(True)
    q, k, v = x[:, :Hq], x[:, Hq:Hq + Hkv], x[:, Hq + Hkv:]
    ref, _ = _attn_ref(q, k, v, causal)
    ref.backward(do.float().view(B, T, Hq, d).transpose(1, 2))
    ref_grad = x.grad.transpose(1, 2).reshape(B * T, W)
    assert not torch.isnan(dqkv.float()).any()
    for name, sl in [("dq", slice(0, Hq * d)), ("dk", slice(Hq * d, (Hq + Hkv) * d)),
                     ("dv", slice((Hq + Hkv) * d, W))]:
        err = rel_err(dqkv[:, sl], ref_grad[:, sl])
        assert err < 3e-2, f"{name} rel err {err}"
    assert ext().status_read(0) == 0


def test_attn_large_score_jump_fwd_bwd():
    """Rows whose last (diagonal) key scores ~200 nats above all earlier keys: the running
    max must move without any exponential overflowing or the row sum underflowing."""
    B, T, Hq, Hkv, d = 1, 1024, 2, 1, 128
    W = (Hq + 2 * Hkv) * d
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = (torch.randn(B * T, W, device="cuda", generator=g) * 0.3)
    for t in (5, 300, 771, 1023):  # q_t . k_t / sqrt(d) ~ 200 for both q heads
        qkv[t, :Hq * d] = 4.0
        qkv[t, Hq * d:(Hq + Hkv) * d] = 4.0
    qkv = qkv.bfloat16()
    o = torch.empty(B * T, Hq * d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, T, device="cuda")
    scale = 1 / math.sqrt(d)
    ext().attn_fwd(qkv, qkv, qkv, 0, Hq * d, (Hq + Hkv) * d, B, T, T, Hq, Hkv, d, o, lse, scale, True, 0)
    x = qkv.float().view(B, T, Hq + 2 * Hkv, d).transpose(1, 2).detach().requires_grad_(True)
    q, k, v = x[:, :Hq], x[:, Hq:Hq + Hkv], x[:, Hq + Hkv:]
    ref, ref_lse = _attn_ref(q, k, v, True)
    assert torch.isfinite(lse).all()
    assert (lse - ref_lse).abs().max().item() < 2e-2
    assert rel_err(o.view(B, T, Hq, d).transpose(1, 2), ref) < 2e-2
    do = torch.randn(B * T, Hq * d, device="cuda", generator=g).bfloat16()
    dqkv = torch.full((B * T, W), float("nan"), device="cuda", dtype=torch.bfloat16)
    dq_acc = torch.empty(B * T, Hq * d, device="cuda")
    scr = torch.empty(ext().attn_bwd_scratch_numel(B, Hq, T), device="cuda")
    ext().attn_bwd(qkv, qkv, qkv, o, do, 0, Hq * d, (Hq + Hkv) * d, lse, B, T, Hq, Hkv, d,
                   dqkv, 0, dqkv, Hq * d, dqkv, (Hq + Hkv) * d, dq_acc, scr, scale, True)
    ref.backward(do.float().view(B, T, Hq, d).transpose(1, 2))
    ref_grad = x.grad.transpose(1, 2).reshape(B * T, W)
    assert torch.isfinite(dqkv.float()).all()
    assert rel_err(dqkv, ref_grad) < 3e-2
    assert ext().status_read(0) == 0


def test_exp2_poly_matches_cuda_exp2():
    x = torch.cat([torch.linspace(-126, 10, 2_000_001, device="cuda"), torch.rand(100000, device="cuda") * -20])
    y = torch.empty_like(x)
    ext().exp2_poly(x, y)
    ref = torch.exp2(x.double())
    rel = ((y.double() - ref).abs() / ref).max().item()
    assert rel < 2e-4, rel  # far below the bf16 resolution (3.9e-3) of P
