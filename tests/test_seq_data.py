"""Packing of jagged sequences (CPU)."""
from flare_b200.data.synthetic import SeqSyntheticData
from flare_b200.ops.attention import pack_offsets


def test_pack_offsets_alignment():
    o, valid = pack_offsets([3, 9, 8, 1])
    assert o.tolist() == [0, 8, 24, 32, 40]
    assert valid.sum().item() == 21 and valid[:3].all() and not valid[3:8].any()


def test_seq_batch_targets_and_kjt():
    d = SeqSyntheticData(5, item_rows=1000, side_rows=50, min_len=3, max_len=40, negatives=16, world=2, rank=0)
    b = d.next()
    offs = b.seq_offsets.tolist()
    assert all(o % 8 == 0 for o in offs) and offs[-1] == b.tokens
    tr = b.target_row.tolist()
    for t, x in enumerate(tr):
        if x >= 0:
            assert x == t + 1
            s = max(i for i in range(len(offs) - 1) if offs[i] <= t)
            assert x < offs[s + 1]
    F, B = 5, d.T_cap + 16
    assert b.emb_offsets.numel() == F * B + 1
    lens = (b.emb_offsets[1:] - b.emb_offsets[:-1]).view(F, B)
    assert int(lens[0, d.T_cap:].sum()) == 16 and int(lens[1:, d.T_cap:].sum()) == 0
    assert int(lens[0, :d.T_cap].sum()) == int(lens[1, :d.T_cap].sum())
    # the global count covers both ranks: the other rank derives the same number
    other = SeqSyntheticData(5, item_rows=1000, side_rows=50, min_len=3, max_len=40, negatives=16, world=2, rank=1)
    assert int(other.next().num_valid) == int(b.num_valid)
