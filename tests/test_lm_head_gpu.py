"""LM head + cross-entropy: the row-chunked variant (no [tokens, vocab] logits buffer,
logits recomputed in the backward) against the single fused pass, and both against an
fp32 reference; with main_grad accumulation like the trainer uses."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N,H,V,rows", [(1000, 256, 5000, 384), (4096, 512, 8192, 1024)])
def test_chunked_lm_head_ce_matches_fused_and_fp32(N, H, V, rows):
    from tinytron_b200 import ops
    from tinytron_b200.ops import check_status

    g = torch.Generator(device="cuda").manual_seed(N)
    h0 = torch.randn(N, H, device="cuda", generator=g).bfloat16()
    w0 = torch.randn(V, H, device="cuda", generator=g) * 0.05
    t = torch.randint(0, V, (N,), device="cuda", generator=g)
    t[::11] = -100
    res = {}
    for chunk in (0, rows):
        h = h0.clone().requires_grad_(True)
        w = w0.clone().requires_grad_(True)
        loss = ops.lm_head_ce_sum(h, w, t, -100, chunk_rows=chunk)
        (loss * 0.5).backward()
        res[chunk] = (loss.detach(), h.grad.float(), w.grad.float())
    torch.cuda.synchronize()
    check_status()
    hf = h0.float().requires_grad_(True)
    wf = w0.bfloat16().float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(hf @ wf.t(), t, ignore_index=-100, reduction="sum")
    (ref * 0.5).backward()
    rel = lambda a, b: ((a - b).norm() / b.norm()).item()  # noqa: E731
    for chunk, (loss, dh, dw) in res.items():
        assert abs(loss.item() - ref.item()) < 1e-2 * abs(ref.item()), chunk
        assert rel(dh, hf.grad) < 2e-2 and rel(dw, wf.grad) < 2e-2, chunk
    # the chunked pass reproduces the fused one (same kernels, same row order)
    assert torch.allclose(res[rows][0], res[0][0], rtol=1e-5)
    assert rel(res[rows][1], res[0][1]) < 1e-3 and rel(res[rows][2], res[0][2]) < 1e-3
