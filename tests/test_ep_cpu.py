"""Expert-parallel bookkeeping on the CPU: receive layouts and expert-block checkpoints."""
import numpy as np
import torch

from atomic_ai_hybrid_b200.ckpt.manager import _lookup
from atomic_ai_hybrid_b200.parallel.ep import receive_layout


def test_receive_layout_partitions_rows():
    rng = np.random.default_rng(0)
    W, E = 4, 16
    El = E // W
    cnt = rng.integers(0, 300, size=(W, E))
    cnt[1, 5] = 0
    layouts = [receive_layout(cnt, r, El) for r in range(W)]
    for r in range(W):  # receiver r: every source's block of every local expert, disjoint, padded segments
        _, off, seg = layouts[r]
        assert off[0] == 0 and all((off[1:] - off[:-1]) % 128 == 0)
        np.testing.assert_array_equal(seg, cnt[:, r * El:(r + 1) * El].sum(0))
        used = np.zeros(off[-1], dtype=np.int64)
        for s in range(W):
            base = layouts[s][0]
            for j in range(El):
                e = r * El + j
                lo, hi = base[e], base[e] + cnt[s, e]
                assert off[j] <= lo and hi <= off[j] + seg[j]
                used[lo:hi] += 1
        for j in range(El):
            assert (used[off[j]:off[j] + seg[j]] == 1).all()
            assert (used[off[j] + seg[j]:off[j + 1]] == 0).all()


def test_expert_block_lookup_assembles_ranges():
    full = torch.arange(8 * 3, dtype=torch.float32).view(8, 3)
    blocks = {f"moe/routed_w1#experts[{lo}:{lo + 2}]": full[lo:lo + 2] for lo in range(0, 8, 2)}
    assert torch.equal(_lookup(blocks, "moe/routed_w1", None), full)
    assert torch.equal(_lookup(blocks, "moe/routed_w1", (2, 6)), full[2:6])
    assert torch.equal(_lookup({"moe/routed_w1": full}, "moe/routed_w1", (4, 8)), full[4:8])
    del blocks["moe/routed_w1#experts[4:6]"]
    assert _lookup(blocks, "moe/routed_w1", (2, 8)) is None
    assert _lookup(blocks, "moe/other", None) is None
