"""Tree replicas: a second DeviceTree fed only with the owner's deltas
(TreeReplicaSync.share, the arrays that a broadcast would carry) answers
match_prefix exactly like the owner, on the reference's recorded stress
queries, with deltas taken while the tree grows (full deltas after resizes
and rehashes, incremental ones between)."""

import json

import numpy as np
import pytest
import torch

from agentkv_b200 import AgentKVPool, PoolConfig
from agentkv_b200 import workloads as W
from agentkv_b200.device_tree import DeviceTree, match_batch
from agentkv_b200.sharded_tree import TreeReplicaSync

pytestmark = pytest.mark.gpu


def test_replica_from_deltas_matches_reference(golden_dir):
    g = np.load(golden_dir / "match_small.npz")
    spec = W.MatchSpec(**json.loads(str(g["spec"])))
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)
    cfg = PoolConfig(total_blocks=int(g["total_blocks"]), block_size=16, num_layers=1, num_kv_heads=1,
                     head_dim=1, dtype="float16", device="meta")
    pool = AgentKVPool(config=cfg)
    owner = pool._tree._dev_tree
    sync = TreeReplicaSync(owner)
    replica = DeviceTree(owner.device)
    replica.as_replica()
    kinds = []
    runs_seen = 0
    queries = W.match_queries(spec, corpus, prefixes, batch=0, n=len(g["node"]))
    for i, seq in enumerate(corpus):
        h = pool.create_root(seq)
        pool.allocate_blocks(h, -(-len(seq) // 16) - len(pool.get_block_ids(h)))
        share = (len(seq) // 16) * 16 - h.shared_match_len
        if share > 0:
            pool.commit_prefix(h, share)
        if i % 37 == 0 or i == len(corpus) - 1:
            owner.build_runs()  # current runs on every share, so each one travels
            d = sync.share()
            if d is not None:
                kinds.append("commands" if "commands" in d else ("full" if d["full"] else "rows"))
                replica.apply_shared(d)
                if "run_head" in d:
                    replica.set_runs(d["run_head"], d["runs"])
                    runs_seen += 1
            if i % 111 == 0:
                # mid-build: the replica answers like the owner
                n0, l0 = match_batch(owner, queries[:64], 16)
                n1, l1 = match_batch(replica, queries[:64], 16)
                np.testing.assert_array_equal(n1, n0)
                np.testing.assert_array_equal(l1, l0)
    # the whole arrays after a resize, else the owner tree's insert commands
    assert "full" in kinds and kinds.count("commands") > len(kinds) // 2, kinds
    assert runs_seen > 1 and replica.d_run_head is not None  # the owner's runs reached the replica
    node, mlen, cmp_ = match_batch(replica, queries, 16, with_compared=True)
    np.testing.assert_array_equal(node, g["node"])
    np.testing.assert_array_equal(mlen, g["len"])
    _, _, cmp_owner = match_batch(owner, queries, 16, with_compared=True)
    np.testing.assert_array_equal(cmp_, cmp_owner)
    # the arrays themselves are identical
    n = owner.n_tokens
    assert torch.equal(replica.d_tokens[:n], owner.d_tokens[:n])
    assert torch.equal(replica.d_slots, owner.d_slots)
    assert torch.equal(replica.d_off, owner.d_off) and torch.equal(replica.d_len, owner.d_len)
    # nothing pending: share() says so
    assert sync.share() is None


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_device_built_tree_changes_over_reference_traces(golden_dir, seed):
    """akv_tree_commands on the GPU: the replica applies the host tree's
    inserts and prunes itself.  Over the reference's recorded tree traces,
    after every commit, free and create, the device arrays (tokens, edge
    ranges, hash slots) equal the host mirror's byte for byte, with most
    uploads done as commands."""
    from test_host_replays import replay_tree_trace_with_array_checks

    _, n_cmd, checked = replay_tree_trace_with_array_checks(golden_dir, seed, torch.device("cuda", 0))
    assert checked > 50 and n_cmd > 20, (checked, n_cmd)


def test_device_built_tree_changes_under_random_churn():
    """The same under random commits and frees reaching every insert branch
    (new leaf, descent, exact re-commit, split off and on block boundaries,
    split == 0 overwrite) and many prunes: byte-equal arrays after every
    step."""
    from agentkv_b200 import AgentKVPool, PoolConfig
    from tree_churn import churn

    for seed in range(3):
        pool = AgentKVPool(config=PoolConfig(total_blocks=400, block_size=4, num_layers=1, num_kv_heads=1,
                                             head_dim=2, dtype="float16", device="meta", epoch_interval=7))
        tree = pool._tree
        dt = tree._dev_tree
        before = dt.command_uploads

        def check(step):
            dt.flush()
            k = dt.n_tokens
            assert np.array_equal(dt.d_tokens[:k].cpu().numpy(), dt.h_tokens[:k]), (seed, step)
            assert np.array_equal(dt.d_off.cpu().numpy(), dt.h_off), (seed, step)
            assert np.array_equal(dt.d_len.cpu().numpy(), dt.h_len), (seed, step)
            assert np.array_equal(dt.d_slots.cpu().numpy(), dt.h_slots), (seed, step)

        churn(tree, np.random.default_rng(seed), 400, check)
        dt.check()
        assert dt.command_uploads - before > 100
