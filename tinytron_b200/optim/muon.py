"""Muon (reference: tinytron/optim/muon.py:4-97, after K. Jordan's Muon).

Quintic Newton-Schulz iteration with coefficients (3.4445, -4.7750, 2.0315) in
bf16, Frobenius pre-normalisation, transposed when rows > cols; Nesterov momentum
via lerp; update scaled by sqrt(max(1, rows/cols)); decoupled weight decay; a
built-in Adam branch for non-matrix parameters.  On CUDA the three matmuls per
iteration (X X^T, A A^T — A is symmetric — and B X) run on the tcgen05 GEMM.
"""
from __future__ import annotations

import torch

NS_COEFFS = (3.4445, -4.7750, 2.0315)


def _ns_iteration_cuda(X: torch.Tensor, steps: int) -> torch.Tensor:
    from tinytron_b200.ops import _ext

    C = _ext.load()
    a, b, c = NS_COEFFS
    r, n = X.shape
    A = torch.empty(r, r, device=X.device, dtype=torch.bfloat16)
    A2 = torch.empty_like(A)
    BX = torch.empty_like(X)
    for _ in range(steps):
        C.gemm(X, X, A, False, False, False, 1.0, None, 0)      # A = X X^T
        C.gemm(A, A, A2, False, False, False, 1.0, None, 0)     # A^2 = A A^T (A symmetric)
        B = torch.add(A, A2, alpha=c / b).mul_(b)               # b*A + c*A^2
        C.gemm(B, X, BX, False, True, False, 1.0, None, 0)      # B X
        X = torch.add(BX, X, alpha=a)                           # a*X + B X
    return X


def zeropower_via_newtonschulz5(G: torch.Tensor, steps: int) -> torch.Tensor:
    assert G.ndim >= 2
    a, b, c = NS_COEFFS
    X = G.bfloat16()
    transposed = G.size(-2) > G.size(-1)
    if transposed:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    if X.is_cuda and X.ndim == 2 and X.size(-1) % 8 == 0 and X.size(-2) % 8 == 0:
        X = _ns_iteration_cuda(X.contiguous(), steps)
    else:
        for _ in range(steps):
            A = X @ X.mT
            B = b * A + c * A @ A
            X = a * X + B @ X
    if transposed:
        X = X.mT
    return X


def muon_update(grad, momentum, beta=0.95, ns_steps=5, nesterov=True):
    momentum.lerp_(grad, 1 - beta)
    update = grad.lerp_(momentum, beta) if nesterov else momentum
    if update.ndim == 4:
        update = update.view(len(update), -1)
    update = zeropower_via_newtonschulz5(update, steps=ns_steps)
    update *= max(1, update.size(-2) / update.size(-1)) ** 0.5
    return update


def adam_update(grad, buf1, buf2, step, betas, eps):
    buf1.lerp_(grad, 1 - betas[0])
    buf2.lerp_(grad.square(), 1 - betas[1])
    buf1c = buf1 / (1 - betas[0] ** step)
    buf2c = buf2 / (1 - betas[1] ** step)
    return buf1c / (buf2c.sqrt() + eps)


class Muon(torch.optim.Optimizer):
    def __init__(self, param_groups):
        for group in param_groups:
            assert "use_muon" in group
            if group["use_muon"]:
                group["params"] = sorted(group["params"], key=lambda x: x.size(), reverse=True)
                group.setdefault("lr", 0.02)
                group.setdefault("momentum", 0.95)
                group.setdefault("weight_decay", 0)
                group.pop("use_adam", None)
                assert set(group) == {"params", "lr", "momentum", "weight_decay", "use_muon"}
            elif group.get("use_adam", False):
                group.setdefault("lr", 3e-4)
                group.setdefault("betas", (0.9, 0.95))
                group.setdefault("eps", 1e-10)
                group.setdefault("weight_decay", 0)
                group.pop("use_adam", None)
                assert set(group) == {"params", "lr", "betas", "eps", "weight_decay", "use_muon"}
            else:
                raise NotImplementedError
        super().__init__(param_groups, dict())

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                state = self.state[p]
                if group["use_muon"]:
                    if not state:
                        state["momentum_buffer"] = torch.zeros_like(p)
                    upd = muon_update(p.grad, state["momentum_buffer"], beta=group["momentum"])
                    p.mul_(1 - group["lr"] * group["weight_decay"])
                    p.add_(upd.reshape(p.shape), alpha=-group["lr"])
                else:
                    if not state:
                        state["exp_avg"] = torch.zeros_like(p)
                        state["exp_avg_sq"] = torch.zeros_like(p)
                        state["step"] = 0
                    state["step"] += 1
                    upd = adam_update(p.grad, state["exp_avg"], state["exp_avg_sq"], state["step"], group["betas"],
                                      group["eps"])
                    p.mul_(1 - group["lr"] * group["weight_decay"])
                    p.add_(upd, alpha=-group["lr"])
        return loss
