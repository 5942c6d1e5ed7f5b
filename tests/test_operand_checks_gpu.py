"""Host-side operand checks and device-side index bounds fail loudly without touching
memory they should not: a host tensor or a misaligned output is rejected before any
launch, and a decode bookkeeping step past the last token column records kBadIndex in
the status word instead of writing out of range (the context stays usable)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

K_BAD_INDEX = 8


def _C():
    from tinytron_b200.ops import _ext

    return _ext.load()


def test_host_tensor_rejected_before_launch():
    a = torch.ones(128, 64, device="cuda", dtype=torch.bfloat16)
    b = torch.ones(256, 64, device="cuda", dtype=torch.bfloat16)
    c = torch.zeros(128, 256, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="tensor operands must be CUDA tensors"):
        _C().gemm(a, b.cpu(), c)
    with pytest.raises(RuntimeError, match="tensor operands must be CUDA tensors"):
        _C().skinny_linear(a[:4], b, c[:4].cpu())
    assert (c == 0).all()  # nothing ran
    _C().gemm(a, b, c)  # the same call with device operands runs: c = a b^T = 64 everywhere
    torch.cuda.synchronize()
    assert (c.float() == 64.0).all()
    assert _C().status_read(torch.cuda.current_device()) == 0


def test_misaligned_split_sum_output_rejected():
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(4, 512, device="cuda", generator=g).bfloat16()
    w = torch.randn(2048, 512, device="cuda", generator=g).bfloat16()
    buf = torch.empty(4 * 2048 + 8, device="cuda", dtype=torch.bfloat16)
    out = buf[1:1 + 4 * 2048].view(4, 2048)  # 2-byte offset: not 8-byte aligned
    with pytest.raises(RuntimeError):
        _C().skinny_linear(x, w, out)


def test_decode_advance_step_past_the_end_sets_bad_index():
    from tinytron_b200.ops import check_status

    C = _C()
    dev = torch.cuda.current_device()
    B, P, total = 3, 5, 8
    tokens = torch.full((B, total + 4), -7, dtype=torch.long, device="cuda")
    view = tokens[:, :total]  # the columns decode_advance may write; the rest is a guard band
    nxt = torch.tensor([11, 12, 13], dtype=torch.long, device="cuda")
    tok_in = torch.zeros(B, dtype=torch.long, device="cuda")
    rng = torch.tensor([1234, 0], dtype=torch.long, device="cuda")
    for step in range(total - P):  # in range: columns P .. total-1
        C.decode_advance(nxt + step, view, P, tok_in, rng, None, None)
    torch.cuda.synchronize()
    check_status()
    assert int(rng[1]) == total - P
    C.decode_advance(nxt, view, P, tok_in, rng, None, None)  # step = total - P: column `total` is past the end
    torch.cuda.synchronize()
    assert int(C.status_read(dev)) == K_BAD_INDEX
    C.status_clear(dev)
    assert (tokens[:, total:] == -7).all()  # nothing written past the end
    for step in range(total - P):
        assert (tokens[:, P + step] == nxt + step).all()
    assert (tokens[:, :P] == -7).all()
    assert int(C.status_read(dev)) == 0
