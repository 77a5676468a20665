"""The draft tree the attention kernels consume (SpeculativeDraftTree,
mtp_engine.py:635-719): the package's host mirror and the oracle's
restatement against the reference's own outputs in tests/golden/draft_tree.npz
(parent index, ancestor mask, linear layout, active node count).  CPU only."""

import numpy as np
import pytest
import torch

from mtp_draft_tree import SpeculativeDraftTree
from oracle import mtp_oracle as O

CASES = [(16, 4, "tree"), (4, 8, "tree"), (4, 8, "trunk"), (4, 2, "tree"), (3, 8, "tree"),
         (5, 3, "tree"), (8, 4, "tree"), (1, 4, "tree"), (1, 1, "trunk"), (6, 1, "tree"),
         (7, 2, "trunk"), (2, 3, "tree")]


@pytest.mark.parametrize("depth,br,mode", CASES)
def test_matches_reference(golden, depth, br, mode):
    g = golden("draft_tree.npz")
    key = f"{mode}_{depth}_{br}"
    t = SpeculativeDraftTree(depth, br, mode)
    assert t.parent.dtype == torch.int32 and t.tree_mask.dtype == torch.float32
    assert t.max_nodes == depth * br
    np.testing.assert_array_equal(t.parent.numpy(), g[key + "_parent"])
    np.testing.assert_array_equal(t.tree_mask.numpy(), g[key + "_mask"])
    do, bo = t.build_linear_layout()
    assert do.dtype == torch.int32 and bo.dtype == torch.int32
    np.testing.assert_array_equal(do.numpy(), g[key + "_depth_offsets"])
    np.testing.assert_array_equal(bo.numpy(), g[key + "_branch_offsets"])
    assert t.active_node_count() == int(g[key + "_active"])
    np.testing.assert_array_equal(t.linear_parent.numpy(), g[key + "_parent"])


@pytest.mark.parametrize("depth,br,mode", CASES)
def test_oracle_matches_reference(golden, depth, br, mode):
    g = golden("draft_tree.npz")
    key = f"{mode}_{depth}_{br}"
    parent, mask = O.draft_tree(depth, br, mode)
    np.testing.assert_array_equal(parent, g[key + "_parent"])
    np.testing.assert_array_equal(mask, g[key + "_mask"])


def test_config4_tree():
    t = SpeculativeDraftTree(16, 4, "tree")
    assert t.active_node_count() == 64
    depth = np.zeros(64, int)
    p = t.parent.numpy()
    for n in range(1, 64):
        depth[n] = depth[p[n]] + 1
    assert np.bincount(depth).tolist() == [1, 4, 16, 43]
    # a node's row of the mask lists exactly its root path
    for n in range(64):
        path, m = {n}, n
        while p[m] >= 0:
            m = int(p[m])
            path.add(m)
        assert set(np.nonzero(t.tree_mask[n].numpy())[0].tolist()) == path


def test_bad_arguments():
    with pytest.raises(ValueError):
        SpeculativeDraftTree(0, 4)
    with pytest.raises(ValueError):
        SpeculativeDraftTree(4, 2, mode="chain")
