"""Replica groups and owners for TP ranks that hold identical KV (host only)."""
import pytest

from tutti_b200.parallel.fanout import owner_of
from tutti_b200.parallel.replica_layout import (read_plan, replica_group, replica_owner,
                                                validate_replica_io)


def test_duplicated_heads_form_adjacent_groups():
    # 4 KV heads at TP8: each head on a pair of ranks
    assert [replica_group(r, 8, 4) for r in range(8)] == [(0, 1), (0, 1), (2, 3), (2, 3), (4, 5), (4, 5),
                                                          (6, 7), (6, 7)]
    # 1 KV head at TP8: all ranks identical
    assert replica_group(5, 8, 1) == tuple(range(8))
    # enough heads: rank-local
    assert replica_group(3, 8, 8) == (3,)


def test_replicated_caches_and_dcp():
    assert replica_group(3, 8, 8, kind="index") == tuple(range(8))
    assert replica_group(3, 8, 4, kind="latent", dcp=2) == (1, 3, 5, 7)
    assert replica_group(2, 8, 4, kind="main", dcp=2) == (2,)


def test_owner_rule_matches_key_prefix_and_spreads_reads():
    keys = [bytes([i]) * 16 for i in range(64)]
    g = (4, 5)
    owners = [replica_owner(k, g) for k in keys]
    assert set(owners) == {4, 5}
    assert replica_owner(keys[3], tuple(range(8))) == owner_of(keys[3], 8)
    plan = read_plan(keys, 5, 8, 4)
    assert all(o in (4, 5) for _, o in plan) and any(o == 5 for _, o in plan)


@pytest.mark.parametrize("kw,msg", [(dict(tp=16, kv_heads=8), "single-node"), (dict(tp=8, kv_heads=4, dp=2), "DP=1"),
                                    (dict(tp=8, kv_heads=4, dcp=4), "DCP"), (dict(tp=8, kv_heads=3), "evenly")])
def test_validation_rejects_unsupported_layouts(kw, msg):
    with pytest.raises(ValueError, match=msg):
        validate_replica_io(**kw)
    validate_replica_io(tp=8, kv_heads=4, dcp=2)
