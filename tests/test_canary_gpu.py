"""Sanitizer substitutes (memory checking without compute-sanitizer).

* Guard bands: every output buffer is the middle of a larger allocation whose head and
  tail hold a sentinel bit pattern; a kernel that writes out of bounds changes them.
* Poisoned receive buffers: outputs start as NaN (or the sentinel), so an element a
  kernel forgot to write shows up, instead of passing by chance with stale zeros.

Applied to the GEMM epilogues (plain, fused axpby, symmetric mirror), the fused norm,
the cross-entropy kernel, the attention forward output, the MoE combine and the
symmetric-heap collectives (graph-safe all-reduce, fused Ulysses exchange) on emulated
ranks, at ragged sizes where bounds handling matters.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

_GUARD = 4096  # elements on each side


class Guarded:
    """A ``shape`` tensor carved from the middle of a buffer with sentinel guard bands."""

    def __init__(self, shape, dtype, fill=float("nan")):
        n = 1
        for s in shape:
            n *= s
        self.buf = torch.empty(n + 2 * _GUARD, device="cuda", dtype=dtype)
        self.bits = self.buf.view(torch.int16 if dtype in (torch.bfloat16, torch.float16) else torch.int32)
        self.bits.fill_(0x5A5A if self.bits.dtype == torch.int16 else 0x5A5A5A5A)
        self.t = self.buf[_GUARD:_GUARD + n].view(shape)
        self.t.fill_(fill)

    def check(self, name="out"):
        torch.cuda.synchronize()
        sentinel = 0x5A5A if self.bits.dtype == torch.int16 else 0x5A5A5A5A
        head, tail = self.bits[:_GUARD], self.bits[-_GUARD:]
        assert bool((head == sentinel).all()), f"{name}: write before the buffer"
        assert bool((tail == sentinel).all()), f"{name}: write past the buffer"
        assert not bool(torch.isnan(self.t.float()).any()), f"{name}: element left unwritten"


def _C():
    from tinytron_b200.ops import _ext

    return _ext.load()


@pytest.mark.parametrize("M,N,K", [(200, 328, 96), (1000, 136, 520), (384, 2056, 264)])
def test_gemm_epilogues_stay_in_bounds(M, N, K):
    C = _C()
    g = torch.Generator(device="cuda").manual_seed(M)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    out = Guarded((M, N), torch.bfloat16)
    C.gemm(a, b, out.t, False, False, False, 1.0, None, 0)
    out.check("gemm bf16")
    f32 = Guarded((M, N), torch.float32, fill=0.0)
    C.gemm(a, b, f32.t, False, False, True, 1.0, None, 0)  # fp32 accumulate
    f32.check("gemm fp32 acc")
    add = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    ax = Guarded((M, N), torch.bfloat16)
    C.gemm_axpby(a, b, ax.t, False, 1.0, add, 0.5, False, 1)
    ax.check("gemm axpby")
    sym = Guarded((M, M), torch.bfloat16)
    C.gemm_axpby(a, a, sym.t, False, 1.0, None, 0.0, True, 1)  # mirrored stores
    sym.check("gemm symmetric")


def test_norm_and_cross_entropy_stay_in_bounds():
    C = _C()
    M, D, V = 333, 1032, 5000
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(M, D, device="cuda", generator=g)
    w = torch.rand(D, device="cuda", generator=g) + 0.5
    h = Guarded((M, D), torch.bfloat16)
    rstd = Guarded((M,), torch.float32)
    C.add_rmsnorm_fwd(x, None, w, None, h.t, rstd.t, 1e-5)
    h.check("rmsnorm h")
    rstd.check("rmsnorm rstd")
    logits = torch.randn(M, V, device="cuda", generator=g).bfloat16()
    tgt = torch.randint(0, V, (M,), device="cuda", generator=g)
    tgt[::7] = -100
    loss = Guarded((M,), torch.float32)
    lse = Guarded((M,), torch.float32)
    C.cross_entropy_fwd(logits, tgt, loss.t, lse.t, -100, False)
    loss.check("ce loss")
    lse.check("ce lse")


def test_attention_output_stays_in_bounds():
    import math

    C = _C()
    B, T, Hq, Hkv, d = 2, 300, 4, 2, 128
    g = torch.Generator(device="cuda").manual_seed(2)
    qkv = torch.randn(B * T, (Hq + 2 * Hkv) * d, device="cuda", generator=g).bfloat16()
    o = Guarded((B * T, Hq * d), torch.bfloat16)
    lse = Guarded((B, Hq, T), torch.float32)
    C.attn_fwd(qkv, qkv, qkv, 0, Hq * d, (Hq + Hkv) * d, B, T, T, Hq, Hkv, d, o.t, lse.t, 1 / math.sqrt(d), True, 0)
    o.check("attn o")
    lse.check("attn lse")


def test_moe_combine_stays_in_bounds():
    from tinytron_b200 import ops

    N, E, k, H, I = 77, 16, 4, 256, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(N, H, device="cuda", generator=g).bfloat16()
    sel = torch.topk(torch.randn(N, E, device="cuda", generator=g), k, -1).indices.to(torch.int32)
    w = torch.softmax(torch.randn(N, k, device="cuda", generator=g), -1)
    Wg, Wu = (torch.randn(E, I, H, device="cuda", generator=g) * 0.05 for _ in range(2))
    Wd = torch.randn(E, H, I, device="cuda", generator=g) * 0.05
    with torch.no_grad():
        y = ops.moe_experts(x, sel, w, Wg, Wu, Wd)
        part = ops.moe_experts_local(x, sel, w, Wg[:8], Wu[:8], Wd[:8], 0)
    torch.cuda.synchronize()
    assert not torch.isnan(y.float()).any() and not torch.isnan(part.float()).any()


def test_heap_collectives_write_every_element_and_stay_in_bounds():
    from tinytron_b200.parallel.symm import SymmetricHeap

    C = _C()
    W, n = 4, 8 * 1000 + 8
    heaps = SymmetricHeap.create_emulated(2 * n * 2 + 8192, W)
    slots = [h.replay_slots(n * 2) for h in heaps]
    ins = [torch.randn(n, device="cuda").bfloat16() for _ in range(W)]
    outs = [Guarded((n,), torch.bfloat16) for _ in range(W)]
    for h, (buf, sb), x in zip(heaps, slots, ins):
        h.replay_publish(buf, sb, x)
    for h, (buf, sb), o in zip(heaps, slots, outs):
        h.replay_reduce(buf, sb, o.t)
    for r, o in enumerate(outs):
        o.check(f"all-reduce rank {r}")
    for h in heaps:
        h.close()
    # fused Ulysses exchange (heads -> tokens direction) with ragged batch and length
    B, T, Hq, D = 3, 40, 8, 64
    hq_l, Wc = Hq // W, Hq // W * D
    nb = W * B * T * Wc * 2
    heaps = SymmetricHeap.create_emulated(2 * nb + 8192, W)
    slots = [h.replay_slots(nb) for h in heaps]
    os_ = [torch.randn(B * W * T, Wc, device="cuda").bfloat16() for _ in range(W)]
    for h, (buf, sb), src in zip(heaps, slots, os_):
        C.ul_pack(h.gid, h.offset_of(buf), sb, src, B, T, [W * T, T, 1], Wc, Wc, Wc, [0] * W, [0] * W, [0] * W)
    ys = [Guarded((B * T, Hq * D), torch.bfloat16) for _ in range(W)]
    for h, (buf, sb), y in zip(heaps, slots, ys):
        C.ul_exchange(h.gid, h.offset_of(buf), sb, y.t, B, T, [T, 0, 1], Wc, Wc)
    for r, y in enumerate(ys):
        y.check(f"ulysses rank {r}")
    for h in heaps:
        h.close()
