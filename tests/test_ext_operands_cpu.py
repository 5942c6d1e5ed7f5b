"""Operand checks of the extension's kernel ops that run before any CUDA call: a pageable
host tensor handed to a kernel op is rejected with an error naming the op (instead of a
kernel dereferencing a host pointer), and ops without tensor operands are unaffected.
Runs without a GPU when the extension has been built; skipped otherwise."""
import pytest
import torch


@pytest.fixture(scope="module")
def C():
    from tinytron_b200.ops import _ext

    try:
        return _ext.load()
    except Exception as e:  # not built, or no CUDA runtime libraries to load it
        pytest.skip(f"extension not loadable here: {e}")


def test_host_tensor_operands_are_rejected(C):
    a = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="gemm: tensor operands must be CUDA tensors"):
        C.gemm(a, a, torch.zeros(4, 4, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="sample_tokens: tensor operands must be CUDA tensors"):
        C.sample_tokens(torch.zeros(2, 8), 1.0, 0, 1.0, 0, 0, torch.zeros(2, dtype=torch.long), None, None)
    with pytest.raises(RuntimeError, match="moe_layout: tensor operands must be CUDA tensors"):
        i32 = torch.zeros(8, dtype=torch.int32)
        C.moe_layout(i32, 4, torch.zeros(5, dtype=torch.int32), i32, torch.zeros(1024, dtype=torch.int32), 128, -1)


def test_ops_without_tensor_operands_still_run(C):
    # (P + E * (align - 1)) rounded up to the alignment
    assert C.moe_row_capacity(10, 4, 128) == 640
    assert C.moe_row_capacity(10, 4, 1) == 10
