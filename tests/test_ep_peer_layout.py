"""CPU check of the receive-buffer layout of the peer-memory EP path (ep_peer._layout)
against a brute-force construction: every owner lists its rows expert by expert and,
inside an expert, source rank by source rank."""
import torch

from moe_ops_b200.ep_peer import _layout


def test_layout_matches_brute_force():
    g = torch.Generator().manual_seed(0)
    for W, El in ((2, 4), (3, 2), (4, 1), (1, 5)):
        E = W * El
        counts = torch.randint(0, 7, (W, E), generator=g, dtype=torch.int32)
        counts[0, 0] = 0  # an empty (source, expert) pair
        # owner -> list of (src, e, i) in receive-buffer order
        pos = {}
        for owner in range(W):
            n = 0
            for le in range(El):
                e = owner * El + le
                for src in range(W):
                    for i in range(int(counts[src, e])):
                        pos[(src, e, i)] = n
                        n += 1
        for r in range(W):
            offsets = torch.zeros(E + 1, dtype=torch.int32)
            offsets[1:] = torch.cumsum(counts[r], 0)
            delta, off_local = _layout(counts, offsets, r, W)
            for e in range(E):
                for i in range(int(counts[r, e])):
                    assert int(offsets[e]) + i + int(delta[e]) == pos[(r, e, i)]
            tot = [int(counts[:, r * El + le].sum()) for le in range(El)]
            want = [0]
            for t in tot:
                want.append(want[-1] + t)
            assert off_local.tolist() == want
