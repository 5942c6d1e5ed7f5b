"""tcgen05 GEMM vs a PyTorch fp32 reference of the same op (all operand majors, epilogues)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def ext():
    from tinytron_b200.ops import _ext

    return _ext.load()


def _operands(M, N, K, a_mn, b_mn, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    return A, B, a, b


def _check(out, ref, tol):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err / scale < tol, f"rel err {err / scale:.3e}"


SHAPES = [(128, 256, 64), (256, 512, 128), (296, 200, 136), (1024, 3072, 2048), (136, 1000, 72), (512, 128, 5504)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("bn", [0, 128, 1])  # 1: the CTA-pair (cta_group::2) kernel
def test_gemm_bf16_out(M, N, K, a_mn, b_mn, bn):
    A, B, a, b = _operands(M, N, K, a_mn, b_mn)
    c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ext().gemm(a, b, c, a_mn, b_mn, False, 1.0, None, bn)
    ref = A.float() @ B.float().t()
    _check(c, ref, 1e-2)
    assert ext().status_read(0) == 0


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (1000, 264, 520)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, True)])
@pytest.mark.parametrize("bn", [0, 1])
def test_gemm_fp32_accumulate_alpha(M, N, K, a_mn, b_mn, bn):
    A, B, a, b = _operands(M, N, K, a_mn, b_mn, seed=1)
    c0 = torch.randn(M, N, device="cuda")
    c = c0.clone()
    alpha_t = torch.tensor([0.5], device="cuda")
    ext().gemm(a, b, c, a_mn, b_mn, True, 2.0, alpha_t, bn)
    ref = c0 + (A.float() @ B.float().t())
    _check(c, ref, 1e-5)
    c2 = torch.empty(M, N, device="cuda")
    ext().gemm(a, b, c2, a_mn, b_mn, False, 0.25, None, bn)
    _check(c2, 0.25 * (A.float() @ B.float().t()), 1e-5)


@pytest.fixture(params=[0, 2], ids=["single_cta", "cta_pair"])
def pair_mode(request):
    prev = ext().gemm_pair_mode()
    ext().gemm_set_pair_mode(request.param)
    yield request.param
    ext().gemm_set_pair_mode(prev)


@pytest.mark.parametrize("M,I,K", [(256, 256, 128), (300, 5504 // 8, 256), (1024, 1408, 2048)])
def test_gemm_swiglu(M, I, K, pair_mode):
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(2 * I, K, device="cuda", generator=g) * 0.05).bfloat16()
    out = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(M, 2 * I, device="cuda", dtype=torch.bfloat16)
    ext().gemm_swiglu(x, w, out, gu)
    pre = x.float() @ w.float().t()
    gate, up = pre[:, :I], pre[:, I:]
    ref = torch.nn.functional.silu(gate) * up
    _check(out, ref, 1e-2)
    _check(gu, pre, 1e-2)


@pytest.mark.parametrize("M,D,I", [(256, 256, 256), (300, 128, 704), (1024, 2048, 1408)])
def test_gemm_dswiglu(M, D, I, pair_mode):
    g = torch.Generator(device="cuda").manual_seed(3)
    dy = torch.randn(M, D, device="cuda", generator=g).bfloat16()
    wd = (torch.randn(D, I, device="cuda", generator=g) * 0.05).bfloat16()
    gu = torch.randn(M, 2 * I, device="cuda", generator=g).bfloat16()
    dgu = torch.empty(M, 2 * I, device="cuda", dtype=torch.bfloat16)
    ext().gemm_dswiglu(dy, wd, gu, dgu, 1.0)
    dact = dy.float() @ wd.float()
    gate, up = gu[:, :I].float(), gu[:, I:].float()
    s = torch.sigmoid(gate)
    ref_dg = dact * up * s * (1 + gate * (1 - s))
    ref_du = dact * gate * s
    _check(dgu[:, :I], ref_dg, 2e-2)
    _check(dgu[:, I:], ref_du, 2e-2)


@pytest.mark.parametrize("M,N,K", [(3072, 2048, 8192), (2048, 5504, 4096)])
def test_gemm_splitk_accumulate_deterministic(M, N, K):
    """Weight-gradient shapes that take the split-K pair kernel: fp32 accumulation into an
    existing buffer matches the fp32 reference and is bitwise reproducible."""
    A, B, a, b = _operands(M, N, K, True, True, seed=4)
    c0 = torch.randn(M, N, device="cuda")
    c1, c2 = c0.clone(), c0.clone()
    ext().gemm(a, b, c1, True, True, True, 1.0, None, 0)
    ext().gemm(a, b, c2, True, True, True, 1.0, None, 0)
    ref = c0 + (A.float() @ B.float().t())
    _check(c1, ref, 1e-5)
    assert torch.equal(c1, c2)
    assert ext().status_read(0) == 0


@pytest.mark.parametrize("M,N,K", [(32, 3072, 2048), (32, 2048, 2048), (1, 64, 2048), (64, 2048, 5504), (17, 304, 1000)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True)])
def test_gemm_small_m(M, N, K, a_mn, b_mn):
    """Decode-sized M (one 128-row tile, mostly padding): bf16 output, alpha applied,
    result identical across calls."""
    A, B, a, b = _operands(M, N, K, a_mn, b_mn, seed=5)
    c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    alpha_t = torch.tensor([0.5], device="cuda")
    ext().gemm(a, b, c, a_mn, b_mn, False, 2.0, alpha_t, 0)
    _check(c, A.float() @ B.float().t(), 1e-2)
    c2 = torch.empty_like(c)
    ext().gemm(a, b, c2, a_mn, b_mn, False, 2.0, alpha_t, 0)
    assert torch.equal(c, c2)
    assert ext().status_read(0) == 0
