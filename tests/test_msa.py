"""MiniMax-M3 sparse attention: block max-pooling, top-k + local block selection, broadcast to keys
and the sparse softmax, against hand-worked cases and a per-query loop written from the rules."""
import math

import pytest
import torch

from fak_b200.models.msa import block_scores, key_mask, msa_attention, select_blocks


def test_hand_worked_selection():
    # 10 keys in blocks of 3: blocks {0,1,2} {3,4,5} {6,7,8} {9}; one query at position 7
    key_pos = torch.arange(10)
    sc = torch.tensor([[0.1, 0.9, 0.2, 0.3, 0.3, 0.1, 0.5, 0.4, 5.0, 9.0]])
    q_pos = torch.tensor([7])
    pooled = block_scores(sc, key_pos, q_pos, 3)
    # keys 8 and 9 are in the future: block 2 pools only keys 6, 7; block 3 has no causal key
    assert pooled[0, :3].tolist() == pytest.approx([0.9, 0.3, 0.5]) and pooled[0, 3] == -math.inf
    sel = select_blocks(pooled, topk=1, local=1)
    assert sel[0].tolist() == [True, False, True, False]        # top-1 = block 0, local = block 2
    m = key_mask(sel, key_pos, q_pos, 3)
    assert torch.nonzero(m[0]).flatten().tolist() == [0, 1, 2, 6, 7]


def test_ties_prefer_the_lower_block_and_nan_is_skipped():
    key_pos = torch.arange(8)
    sc = torch.tensor([[1.0, 0.0, 1.0, 0.0, 1.0, float("nan"), 0.0, 0.0]])
    pooled = block_scores(sc, key_pos, torch.tensor([7]), 2)
    assert pooled[0].tolist() == [1.0, 1.0, 1.0, 0.0]
    assert select_blocks(pooled, topk=2, local=0)[0].tolist() == [True, True, False, False]


def test_bad_layouts_fail_closed():
    with pytest.raises(ValueError):
        block_scores(torch.zeros(1, 3), torch.tensor([0, 1, 1]), torch.tensor([2]), 2)
    with pytest.raises(ValueError):
        block_scores(torch.zeros(1, 3), torch.tensor([0, 1, 2]), torch.tensor([2]), 0)


def _loop_reference(q, K, V, scores, q_pos, key_pos, block, topk, local, scale):
    Tq, H, D = q.shape
    g = H // K.shape[1]
    out = torch.zeros(Tq, H, D, dtype=torch.float64)
    for t in range(Tq):
        pooled = {}
        for j, p in enumerate(key_pos.tolist()):
            v = float(scores[t, j])
            if p <= int(q_pos[t]) and not math.isnan(v):
                b = p // block
                pooled[b] = max(pooled.get(b, -math.inf), v)
        cand = sorted(pooled)
        chosen = set(cand[len(cand) - local:] if local else [])
        chosen |= set(sorted(cand, key=lambda b: (-pooled[b], b))[:topk])
        keys = [j for j, p in enumerate(key_pos.tolist()) if p <= int(q_pos[t]) and p // block in chosen]
        for h in range(H):
            k = K[keys, h // g].double()
            s = (k @ q[t, h].double()) * scale
            w = torch.softmax(s, 0)
            out[t, h] = w @ V[keys, h // g].double()
    return out


@pytest.mark.parametrize("block,topk,local", [(4, 2, 1), (8, 1, 2), (3, 0, 2), (16, 4, 0)])
def test_msa_attention_matches_the_per_query_rules(block, topk, local):
    torch.manual_seed(block * 7 + topk)
    Tk, Tq, H, Hk, D = 50, 6, 4, 2, 16
    key_pos = torch.randperm(Tk)            # a shuffled cache layout
    K, V = torch.randn(Tk, Hk, D), torch.randn(Tk, Hk, D)
    q = torch.randn(Tq, H, D)
    q_pos = torch.tensor([5, 17, 23, 31, 44, 49])
    scores = torch.randn(Tq, Tk)
    got, mask = msa_attention(q, K, V, scores, q_pos, key_pos, block, topk, local)
    want = _loop_reference(q, K, V, scores, q_pos, key_pos, block, topk, local, 1.0 / math.sqrt(D))
    assert torch.allclose(got.double(), want, atol=1e-5)
    # the local window always holds the query's own block when local >= 1
    if local:
        own = (key_pos // block) == (q_pos[:, None] // block)
        assert bool((mask | ~(own & (key_pos[None, :] <= q_pos[:, None]))).all())


def _fixed_loop(pooled, q_pos, block, topk, local):
    out = []
    for t in range(pooled.shape[0]):
        qb = int(q_pos[t]) // block
        cands = [(b, float(pooled[t, b])) for b in range(pooled.shape[1]) if pooled[t, b] > -math.inf]
        cands = [(b, math.inf if local and qb - local < b <= qb else s) for b, s in cands]
        cands.sort(key=lambda c: (-c[1], c[0]))
        out.append(sorted(b for b, _ in cands[:topk]))
    return out


@pytest.mark.parametrize("topk,local", [(2, 1), (3, 2), (1, 3), (5, 0)])
def test_fixed_count_selection_displaces_instead_of_adding(topk, local):
    from fak_b200.models.msa import pooled_over_heads, select_blocks_fixed
    torch.manual_seed(topk * 10 + local)
    Tk, block = 40, 4
    key_pos = torch.arange(Tk)
    q_pos = torch.tensor([3, 9, 18, 27, 39])
    scores = torch.randn(5, 3, Tk)                       # 3 index heads
    pooled = pooled_over_heads(scores, key_pos, q_pos, block)
    want = torch.stack([block_scores(scores[:, h], key_pos, q_pos, block) for h in range(3)]).amax(0)
    assert torch.equal(pooled, want)
    sel = select_blocks_fixed(pooled, q_pos, block, topk, local)
    assert [torch.nonzero(r).flatten().tolist() for r in sel] == _fixed_loop(pooled, q_pos, block, topk, local)
    # the count is fixed: min(topk, causal blocks) whatever the local window
    assert sel.sum(1).tolist() == [min(topk, int(q) // block + 1) for q in q_pos]
