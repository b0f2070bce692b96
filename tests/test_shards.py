"""Sequence shards: contiguous, zigzag (ring) and hybrid layouts cover every position exactly once."""

import pytest
import torch

from bridge_b200.tpr.shard import (PaddedSequenceShard, PrefixShard, RangeSequenceShard, iter_valid_sequence_slices,
                                   make_hybrid_sequence_shard, make_ring_sequence_shard, round_up_sequence_length)


@pytest.mark.parametrize("L,cp", [(128, 2), (130, 4), (7, 2), (512, 8)])
def test_zigzag_partition(L, cp):
    seen = []
    for r in range(cp):
        sh = make_ring_sequence_shard(L, cp_rank=r, cp_size=cp)
        seen += sh.physical_global_indices().tolist()
        x = torch.arange(L)
        sel = sh.select(x)
        assert sel.shape[0] == sh.local_length
        for g in range(L):
            if sh.owns(g):
                assert sh.local_to_global(sh.global_to_local(g)) == g
    assert sorted(seen) == list(range(round_up_sequence_length(L, 2 * cp)))


@pytest.mark.parametrize("L,cp,u", [(64, 4, 2), (100, 8, 2), (96, 8, 4)])
def test_hybrid_partition(L, cp, u):
    seen = []
    for r in range(cp):
        seen += make_hybrid_sequence_shard(L, cp_rank=r, cp_size=cp, ulysses_size=u).physical_global_indices().tolist()
    assert sorted(seen) == list(range(len(seen)))


def test_padded_shard_validity():
    phys = PrefixShard.contiguous(8, cp_rank=1, cp_size=2)
    sh = PaddedSequenceShard(6, phys)
    assert sh.valid_local_length == 2 and sh.local_length == 4
    assert sh.global_indices().tolist() == [4, 5, 5, 5]
    assert iter_valid_sequence_slices(sh) == (((4, 6), slice(0, 2)),)
    with pytest.raises(ValueError):
        sh.local_to_global(3)


def test_range_shard_rejects_overlap():
    with pytest.raises(ValueError):
        RangeSequenceShard(10, ((0, 5), (4, 6)), 0, 2)
