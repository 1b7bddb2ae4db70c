"""Property tests (hypothesis) for the layout arithmetic of the parallel paths: pieces of
split tensors, checkpoint pieces across tensor-parallel sizes, and the expert-parallel
receive layout."""
import numpy as np
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from atomic_ai_hybrid_b200.ckpt.manager import _lookup_tp
from atomic_ai_hybrid_b200.parallel.ep import receive_layout
from atomic_ai_hybrid_b200.parallel.tp import shard_tensor, unshard_tensors


@settings(max_examples=60, deadline=None)
@given(st.integers(1, 3), st.sampled_from([1, 2, 4, 8]), st.sampled_from([1, 2]), st.integers(0, 1),
       st.integers(1, 3))
def test_shard_unshard_round_trip(blocks_per_piece, world, parts, dim, other):
    n = blocks_per_piece * world * parts
    shape = (n, other) if dim == 0 else (other, n)
    full = torch.arange(n * other, dtype=torch.float32).view(shape)
    pieces = [shard_tensor(full, dim, parts, world, r) for r in range(world)]
    assert all(p.shape[dim] == n // world for p in pieces)
    assert torch.equal(unshard_tensors(pieces, dim, parts), full)
    # the pieces cover every element exactly once
    seen = torch.cat([p.reshape(-1) for p in pieces]).sort().values
    assert torch.equal(seen, full.reshape(-1).sort().values)


@settings(max_examples=40, deadline=None)
@given(st.sampled_from([1, 2, 4]), st.sampled_from([1, 2, 4]), st.sampled_from([1, 2]), st.integers(0, 1))
def test_checkpoint_pieces_reshard_between_sizes(w_save, w_load, parts, dim):
    n = 8 * parts
    full = torch.randn(n, 3) if dim == 0 else torch.randn(3, n)
    tensors = {f"w#tp[{r}/{w_save},d{dim}p{parts}]": shard_tensor(full, dim, parts, w_save, r) for r in range(w_save)}
    for r in range(w_load):
        got = _lookup_tp(tensors, "w", (dim, parts, r, w_load))
        assert torch.equal(got, shard_tensor(full, dim, parts, w_load, r))


@settings(max_examples=60, deadline=None)
@given(st.sampled_from([1, 2, 4]), st.integers(1, 4), st.data())
def test_receive_layout_partitions(W, El, data):
    E = W * El
    cnt = np.array(data.draw(st.lists(st.lists(st.integers(0, 300), min_size=E, max_size=E), min_size=W, max_size=W)))
    for r in range(W):
        _, off, seg = receive_layout(cnt, r, El)
        assert off[0] == 0 and all(o % 128 == 0 for o in off)
        assert all(off[j + 1] - off[j] >= seg[j] for j in range(El))
        assert list(seg) == [int(cnt[:, r * El + j].sum()) for j in range(El)]
    used = {}
    for s in range(W):
        base, _, _ = receive_layout(cnt, s, El)
        for e in range(E):
            dest = e // El
            rows = set(range(int(base[e]), int(base[e]) + int(cnt[s, e])))
            prev = used.setdefault(dest, set())
            assert not (prev & rows)  # no two sources write the same row of a receive buffer
            prev |= rows
