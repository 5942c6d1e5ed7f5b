"""Host-side expert-parallel routing plan (tinytron_b200.parallel.ep_comm.plan_finish) on CPU.

Every rank's plan is built from the same [world, E] count matrix, as the kernels do after
the count all-gather; the plans must give every (token, slot) pair a distinct row inside
its expert's segment of the owner's receive buffer, keep each source's pairs in token
order, start segments on the alignment the grouped GEMMs need, and agree on every
owner's segment layout.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from tinytron_b200.parallel import ep_comm as epc


def _plans(W, E, N, k, seed):
    g = torch.Generator().manual_seed(seed)
    sels = []
    for _ in range(W):
        logits = torch.randn(N, E, generator=g)
        logits[:, 0] += 1.5  # skew: one popular expert, some experts possibly empty
        sels.append(torch.topk(logits, k, dim=-1).indices.to(torch.int32))
    M = np.stack([torch.bincount(s.reshape(-1).long(), minlength=E).numpy() for s in sels]).astype(np.int64)
    cap = epc.capacity(W, N, k, E // W)
    plans = []
    for r in range(W):
        bufs = SimpleNamespace(world=W, rank=r, E=E, cap=cap)
        counts = torch.from_numpy(M[r]).to(torch.int32)
        plans.append(epc.plan_finish(bufs, sels[r], counts, M))
    return sels, M, plans


@pytest.mark.parametrize("W,E,N,k", [(2, 8, 64, 2), (4, 16, 96, 4), (8, 64, 128, 8), (2, 64, 4096, 8)])
def test_plan_rows_distinct_ordered_and_aligned(W, E, N, k):
    sels, M, plans = _plans(W, E, N, k, seed=W * 7 + E)
    E_l = E // W
    align = 256 if int(M.sum()) >= 256 * E else 128
    for o in range(W):  # owner o: collect every source's pairs that land here
        grp = plans[o].grp_off.numpy()
        assert grp[0] == 0 and all(x % align == 0 for x in grp)
        assert plans[o].total == grp[-1]
        assert plans[o].pair == (align == 256)
        seen = set()
        for s in range(W):
            tgt, dst = plans[s].tgt.numpy(), plans[s].dst.numpy()
            flat = sels[s].reshape(-1).numpy()
            for e_l in range(E_l):
                e = o * E_l + e_l
                idx = np.nonzero(flat == e)[0]  # this source's pairs for expert e, token order
                assert np.all(tgt[idx] == o)
                rows = dst[idx]
                assert np.all(np.diff(rows) == 1) if len(rows) > 1 else True  # contiguous, in token order
                assert np.all((rows >= grp[e_l]) & (rows < grp[e_l + 1]))
                seen.update(rows.tolist())
        assert len(seen) == int(M[:, o * E_l:(o + 1) * E_l].sum())  # no two pairs share a row
        # real rows of each segment come first, padding after
        cnt = plans[o].seg_cnt.numpy()
        assert np.array_equal(cnt, M[:, o * E_l:(o + 1) * E_l].sum(0))


def test_sources_fill_an_expert_segment_in_rank_order():
    sels, M, plans = _plans(4, 16, 96, 4, seed=3)
    E_l = 4
    for o in range(4):
        grp = plans[o].grp_off.numpy()
        for e_l in range(E_l):
            e = o * E_l + e_l
            start = grp[e_l]
            for s in range(4):
                flat = sels[s].reshape(-1).numpy()
                idx = np.nonzero(flat == e)[0]
                if len(idx):
                    assert plans[s].dst.numpy()[idx[0]] == start + M[:s, e].sum()


def test_buffer_layout_includes_return_records():
    # push-mode combine records one int64 return address per receive row
    base = epc.SymmetricHeap.bytes_needed((2 * 8, torch.int32), (100 * 64, torch.bfloat16), (100 * 64, torch.bfloat16))
    assert epc.EPBuffers.nbytes(2, 8, 64, 100) >= base + 100 * 8


def test_push_combine_switch(monkeypatch):
    monkeypatch.delenv("TT_EP_PUSH_COMBINE", raising=False)
    assert not epc.push_combine_enabled()  # pull-combine by default (measured faster)
    monkeypatch.setenv("TT_EP_PUSH_COMBINE", "1")
    assert epc.push_combine_enabled()
