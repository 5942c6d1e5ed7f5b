"""Muon: SGD-momentum whose update is orthogonalised by a quintic Newton-Schulz
iteration (K. Jordan's Muon), with an Adam branch for the parameters that are not
matrices.  Public names, parameter-group keys and defaults follow the reference
(tinytron/optim/muon.py:4-97): ``zeropower_via_newtonschulz5``, ``muon_update``,
``adam_update``, ``Muon``.

B200 design:

* Newton-Schulz on the tcgen05 GEMM with the iteration's arithmetic in the epilogues.
  One iteration X <- a X + (b A + c A^2) X with A = X X^T is three launches:
    1. A  = X X^T              symmetric output: only the 128x128 tiles on or above
                               the diagonal are computed, each stored twice (mirrored);
    2. B  = c A A^T + b A      symmetric again (A A^T = A^2 because A is symmetric), with
                               the "+ b A" fused into the epilogue;
    3. X' = B X + a X          with the "+ a X" fused into the epilogue.
  Against three plain GEMMs plus two elementwise passes this halves the FLOPs of the
  two r x r products and removes every separate elementwise pass over A and X.
* Matrices of one shape are orthogonalised together: their normalised updates are
  stacked along the rows and every GEMM of an iteration is ONE batched launch over the
  whole stack (e.g. all 48 [2048 x 5504] MLP matrices of a 16-layer model), which fills
  the 148 SMs even for small matrices (GQA k/v projections: 2 x 2 tiles each) and
  replaces thousands of per-matrix launches by a few dozen.
* ``DistributedMuon`` (ZeRO-1): each matrix is orthogonalised by exactly one rank of
  its replica group — every rank of DP x SEP for the dense parameters (they are
  identical there after the gradient sync), every DP rank for expert parameters —
  instead of by every replica.  Owners hold contiguous, tensor-aligned ranges of the
  flat parameter buffer balanced by Newton-Schulz cost, keep optimizer state for their
  own tensors only, and publish the updated range with one broadcast per owner.

The CPU path computes the same iteration with plain bf16 matmuls (the published
algorithm; it is the oracle for the kernels).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

NS_COEFFS = (3.4445, -4.7750, 2.0315)


# ----------------------------------------------------------------------------- Newton-Schulz
def _kernel_ok(X: torch.Tensor) -> bool:
    return X.is_cuda and X.dim() == 2 and X.size(0) % 8 == 0 and X.size(1) % 8 == 0


class _NSWorkspace:
    """bf16 buffers for ``batch`` matrices of one shape [r, n] (r <= n), stacked along the
    rows: A, B [batch * r, r] and the ping-pong X [batch * r, n]."""

    def __init__(self, r: int, n: int, device, batch: int = 1):
        self.r, self.n, self.batch = r, n, batch
        self.A = torch.empty(batch * r, r, device=device, dtype=torch.bfloat16)
        self.B = torch.empty(batch * r, r, device=device, dtype=torch.bfloat16)
        self.X = [torch.empty(batch * r, n, device=device, dtype=torch.bfloat16) for _ in range(2)]


def _ns_tcgen05(X0: torch.Tensor, steps: int, ws: _NSWorkspace) -> torch.Tensor:
    """``steps`` iterations on the tcgen05 GEMM for ``ws.batch`` stacked matrices;
    X0: bf16 [batch * r, n] (r <= n), each matrix already normalised.  Three launches
    per iteration for the whole stack.  Returns a workspace buffer holding the result."""
    from tinytron_b200.ops import _ext

    C = _ext.load()
    a, b, c = NS_COEFFS
    src = X0
    for i in range(steps):
        dst = ws.X[i % 2] if src is not ws.X[i % 2] else ws.X[(i + 1) % 2]
        C.gemm_axpby(src, src, ws.A, False, 1.0, None, 0.0, True, ws.batch)   # A = X X^T
        C.gemm_axpby(ws.A, ws.A, ws.B, False, c, ws.A, b, True, ws.batch)      # B = c A^2 + b A
        C.gemm_axpby(ws.B, src, dst, True, 1.0, src, a, False, ws.batch)       # X' = B X + a X
        src = dst
    return src


def _ns_torch(X: torch.Tensor, steps: int) -> torch.Tensor:
    a, b, c = NS_COEFFS
    for _ in range(steps):
        gram = X @ X.mT
        X = a * X + (b * gram + c * gram @ gram) @ X
    return X


def zeropower_via_newtonschulz5(G: torch.Tensor, steps: int, workspace: _NSWorkspace | None = None) -> torch.Tensor:
    """Approximately orthogonalise G (the nearest semi-orthogonal matrix U V^T of its SVD,
    up to the iteration's tolerance) in bf16: Frobenius-normalise, iterate on the wide
    orientation (rows <= cols), transpose back.  Leading dims are batch dims.  With a
    ``workspace`` the result may live in one of its buffers."""
    if G.dim() < 2:
        raise ValueError("Newton-Schulz needs a matrix (or a batch of matrices)")
    tall = G.size(-2) > G.size(-1)
    X = G.bfloat16()
    if tall:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    if _kernel_ok(X):
        r, n = X.shape
        ws = workspace if workspace is not None and workspace.batch == 1 else _NSWorkspace(r, n, X.device)
        X = _ns_tcgen05(X.contiguous(), steps, ws)
    else:
        X = _ns_torch(X, steps)
    return X.mT if tall else X


def _scale_for_shape(rows: int, cols: int) -> float:
    return max(1.0, rows / cols) ** 0.5


def muon_update(grad, momentum, beta=0.95, ns_steps=5, nesterov=True, workspace=None):
    """Momentum EMA (in place), Nesterov look-ahead (written into ``grad``), then the
    orthogonalised direction scaled by sqrt(max(1, rows / cols))."""
    momentum.lerp_(grad, 1 - beta)
    direction = grad.lerp_(momentum, beta) if nesterov else momentum
    if direction.dim() == 4:  # convolution filters: one matrix per output channel
        direction = direction.view(direction.size(0), -1)
    out = zeropower_via_newtonschulz5(direction, steps=ns_steps, workspace=workspace)
    return out * _scale_for_shape(out.size(-2), out.size(-1))


def adam_update(grad, buf1, buf2, step, betas, eps):
    """Bias-corrected Adam direction; ``buf1``/``buf2`` (first/second moments) update in place."""
    b1, b2 = betas
    buf1.lerp_(grad, 1 - b1)
    buf2.lerp_(grad * grad, 1 - b2)
    m_hat = buf1 / (1 - b1 ** step)
    v_hat = buf2 / (1 - b2 ** step)
    return m_hat / (v_hat.sqrt() + eps)


# ----------------------------------------------------------------------------- optimizer
_MUON_KEYS = {"params", "lr", "momentum", "weight_decay", "use_muon"}
_ADAM_KEYS = {"params", "lr", "betas", "eps", "weight_decay", "use_muon"}


class Muon(torch.optim.Optimizer):
    """Parameter groups carry ``use_muon``: True for matrices (lr 0.02, momentum 0.95 by
    default), False with ``use_adam=True`` for the rest (lr 3e-4, betas (0.9, 0.95),
    eps 1e-10).  Weight decay is decoupled in both.  ``step(grad_scale=...)`` multiplies
    every gradient by a (device) scalar first, e.g. a clip coefficient."""

    def __init__(self, param_groups):
        groups = []
        for g in param_groups:
            g = dict(g)
            if "use_muon" not in g:
                raise ValueError("every Muon parameter group needs a 'use_muon' key")
            if g["use_muon"]:
                g.pop("use_adam", None)
                g["params"] = sorted(g["params"], key=lambda t: tuple(t.size()), reverse=True)
                g = {"lr": 0.02, "momentum": 0.95, "weight_decay": 0, **g}
                keys = _MUON_KEYS
            elif g.pop("use_adam", False):
                g = {"lr": 3e-4, "betas": (0.9, 0.95), "eps": 1e-10, "weight_decay": 0, **g}
                keys = _ADAM_KEYS
            else:
                raise NotImplementedError("a Muon parameter group must set use_muon=True or use_adam=True")
            if set(g) != keys:
                raise ValueError(f"unexpected Muon group keys {sorted(set(g) ^ keys)}")
            groups.append(g)
        super().__init__(groups, {})
        self._workspaces: dict[tuple, _NSWorkspace] = {}

    @torch.no_grad()
    def step(self, closure=None, grad_scale: torch.Tensor | None = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        matrices = []
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                if grad_scale is not None:
                    p.grad.mul_(grad_scale)
                if group["use_muon"]:
                    matrices.append((p, group))
                else:
                    self._adam_step(p, group)
        self._muon_steps(matrices)
        return loss

    def _adam_step(self, p, group):
        st = self.state[p]
        if not st:
            st["exp_avg"] = torch.zeros_like(p)
            st["exp_avg_sq"] = torch.zeros_like(p)
            st["step"] = 0
        st["step"] += 1
        upd = adam_update(p.grad, st["exp_avg"], st["exp_avg_sq"], st["step"], group["betas"], group["eps"])
        p.mul_(1 - group["lr"] * group["weight_decay"])
        p.add_(upd, alpha=-group["lr"])

    def _momentum(self, p):
        st = self.state[p]
        if not st:
            st["momentum_buffer"] = torch.zeros_like(p)
        return st["momentum_buffer"]

    def _muon_one(self, p, group):
        upd = muon_update(p.grad, self._momentum(p), beta=group["momentum"])
        p.mul_(1 - group["lr"] * group["weight_decay"])
        p.add_(upd.reshape(p.shape), alpha=-group["lr"])

    def _muon_steps(self, matrices):
        """Matrices of one shape and group are updated together: multi-tensor momentum
        and Nesterov ops, one stacked bf16 buffer, three batched GEMM launches per
        Newton-Schulz iteration for the whole bucket, multi-tensor weight decay + update."""
        buckets: dict[tuple, list] = {}
        for p, g in matrices:
            if p.is_cuda and p.dim() == 2 and p.size(0) % 8 == 0 and p.size(1) % 8 == 0:
                buckets.setdefault((tuple(p.shape), id(g)), []).append((p, g))
            else:
                self._muon_one(p, g)
        for (shape, _), items in buckets.items():
            self._muon_bucket(shape, [p for p, _ in items], items[0][1])

    def _muon_bucket(self, shape, params, group):
        rows, cols = shape
        tall = rows > cols
        r, n = (cols, rows) if tall else (rows, cols)
        nb = len(params)
        key = (r, n, nb, str(params[0].device))
        ws = self._workspaces.get(key)
        if ws is None:
            ws = self._workspaces[key] = _NSWorkspace(r, n, params[0].device, nb)
        grads = [p.grad for p in params]
        moms = [self._momentum(p) for p in params]
        beta = group["momentum"]
        torch._foreach_lerp_(moms, grads, 1 - beta)   # momentum EMA
        torch._foreach_lerp_(grads, moms, beta)       # Nesterov direction (in place, as muon_update)
        X0 = ws.X[0].view(nb, r, n)
        for i, g in enumerate(grads):                 # bf16 [r, n] (wide orientation)
            X0[i].copy_(g.mT if tall else g)
        norms = X0.view(nb, -1).norm(dim=-1)          # Frobenius norm of each bf16 matrix
        X0.div_((norms + 1e-7).view(nb, 1, 1))
        out = _ns_tcgen05(ws.X[0], 5, ws).view(nb, r, n)
        scale = _scale_for_shape(rows, cols)
        torch._foreach_mul_(params, 1 - group["lr"] * group["weight_decay"])
        torch._foreach_add_(params, [o.mT if tall else o for o in out.unbind(0)], alpha=-group["lr"] * scale)


# ----------------------------------------------------------------------------- ZeRO-1
def ns_cost(shape) -> float:
    """Relative cost of one Muon update of a parameter (Newton-Schulz FLOPs for matrices,
    a small per-element cost for everything else)."""
    if len(shape) < 2:
        return float(shape[0] if shape else 1) * 10.0
    rows, cols = shape[0], 1
    for d in shape[1:]:
        cols *= d
    r, n = min(rows, cols), max(rows, cols)
    return 5.0 * (3.0 * r * r * n + r ** 3)


def contiguous_owner_ranges(offsets, costs, n_owners: int, end: int) -> list[tuple[int, int, int, int]]:
    """Split tensors (in buffer order) into ``n_owners`` contiguous runs of roughly equal
    total cost.  Returns per owner (first tensor, last tensor + 1, buffer lo, buffer hi);
    the runs cover the tensors in order and the buffer ranges tile [offsets[0], end)."""
    total = float(sum(costs))
    bounds = [0]
    acc = 0.0
    t = 0
    for k in range(1, n_owners):
        target = total * k / n_owners
        while t < len(costs) and acc + costs[t] / 2 < target:
            acc += costs[t]
            t += 1
        bounds.append(max(t, bounds[-1]))
    bounds.append(len(costs))
    out = []
    for k in range(n_owners):
        i0, i1 = bounds[k], bounds[k + 1]
        lo = offsets[i0] if i0 < len(offsets) else end
        hi = offsets[i1] if i1 < len(offsets) else end
        if k == 0:
            lo = offsets[0] if offsets else end
        out.append((i0, i1, lo, hi))
    return out


class DistributedMuon:
    """ZeRO-1 Muon over a :class:`~tinytron_b200.parallel.buffers.FlatParams`: every
    tensor is updated by one owner of its replica group (see the module docstring), and
    the owners broadcast their contiguous ranges of the flat fp32 buffer afterwards.

    ``dense_group`` spans the ranks holding identical dense parameters (DP x SEP);
    ``expert_group`` the ranks holding identical expert parameters (DP).  Either may be
    None (size 1).  The wrapped ``Muon`` keeps only this rank's tensors in its groups,
    so its state dict holds only the owned state."""

    def __init__(self, optimizer: Muon, flat, dense_group=None, expert_group=None):
        self.optimizer = optimizer
        self.flat = flat
        self.part_assignment = {}
        owner_of = {}
        self._broadcasts = []  # (lo, hi, src global rank, group)
        n_dense = sum(1 for o in flat.offsets if o < flat.dense_numel) if flat.dense_numel < flat.numel \
            else len(flat.params)
        for kind, group, idx in (("dense", dense_group, range(0, n_dense)),
                                 ("expert", expert_group, range(n_dense, len(flat.params)))):
            idx = list(idx)
            if not idx:
                continue
            world = dist.get_world_size(group) if group is not None else 1
            me = dist.get_rank(group) if group is not None else 0
            end = flat.dense_numel if kind == "dense" else flat.numel
            offs = [flat.offsets[i] for i in idx]
            costs = [ns_cost(tuple(flat.params[i].shape)) for i in idx]
            ranges = contiguous_owner_ranges(offs, costs, world, end)
            for owner, (i0, i1, lo, hi) in enumerate(ranges):
                for j in idx[i0:i1]:
                    owner_of[id(flat.params[j])] = (owner, owner == me)
                if world > 1 and hi > lo:
                    src = dist.get_global_rank(group, owner) if group is not None else owner
                    self._broadcasts.append((lo, hi, src, group))
        for gi, g in enumerate(optimizer.param_groups):
            keep = []
            for pi, p in enumerate(g["params"]):
                owner, mine = owner_of.get(id(p), (None, True))
                self.part_assignment[(gi, pi)] = owner  # owner's rank in the tensor's replica group
                if mine:
                    keep.append(p)
            g["params"] = keep

    @property
    def param_groups(self):
        return self.optimizer.param_groups

    def state_dict(self):
        return self.optimizer.state_dict()

    def load_state_dict(self, sd):
        self.optimizer.load_state_dict(sd)

    @torch.no_grad()
    def step(self, grad_scale=None):
        self.optimizer.step(grad_scale=grad_scale)
        for lo, hi, src, group in self._broadcasts:
            dist.broadcast(self.flat.data[lo:hi], src=src, group=group)

    def zero_grad(self, set_to_none: bool = True):
        self.flat.zero_grad()
