"""Static speculative draft tree: the node numbering, parent index and
ancestor mask that the tree attention kernels consume.

Mirrors ``SpeculativeDraftTree`` of the reference engine
(mtp_engine.py:635-719): same constructor, attributes and layout, so a
caller's ``tree.tree_mask`` goes straight into ``fused_tree_attention_paged``
(``tree_mask[n, m] = 1`` when m is n or an ancestor of n) and into the
single-query ``fused_tree_attention`` (one row of it as the key mask).

Nodes are numbered breadth first.  Level 0 is the root (node 0); level d
holds ``n_d = min(n_{d-1} * max_branches, max_nodes - s_d)`` nodes starting
at ``s_d``, and node ``s_d + j`` is child ``j % max_branches`` of node
``s_{d-1} + j // max_branches`` -- the reference builds the same numbering
with a frontier walk (651-669).  ``mode="trunk"`` is a single chain
0 <- 1 <- ... <- depth-1; the nodes after it have no parent.

The layout is built once per tree on the host with whole-array operations
(the ancestor mask by walking every node's parent chain in parallel, one
level per step) and then copied to the device by the caller; it is build
time, not step time.
"""

from typing import Optional, Tuple

import numpy as np
import torch


def _levels(depth: int, max_branches: int, max_nodes: int):
    """(start, size) of each BFS level of the "tree" mode, root first."""
    out = [(0, 1)] if max_nodes > 0 else []
    start, size = 1, 1
    for _ in range(1, depth):
        n = max(0, min(size * max_branches, max_nodes - start))
        out.append((start, n))
        start, size = start + n, n
    return out


class SpeculativeDraftTree:
    """Static draft tree of ``depth * max_branches`` node slots
    (mtp_engine.py:635-650).  ``parent`` int32 ``[max_nodes]`` (-1 for the
    root and unused slots) and ``tree_mask`` float32 ``[max_nodes, max_nodes]``
    live on the host, like the reference's; ``build_linear_layout`` returns
    its tensors on ``device``."""

    def __init__(self, depth: int, max_branches: int = 8, mode: str = "tree",
                 device: Optional[torch.device] = None):
        if mode not in ("tree", "trunk"):
            raise ValueError(f"mode must be 'tree' or 'trunk', got {mode!r}")
        self.depth = int(depth)
        self.max_branches = int(max_branches)
        self.mode = mode
        self.device = device or torch.device("cpu")
        self.max_nodes = self.depth * self.max_branches
        if self.max_nodes < 1:
            # the reference fails here too (its mask[0, 0] store, 680)
            raise ValueError(f"depth * max_branches must be >= 1, got {self.depth} * {self.max_branches}")
        self.parent = self._build_parent_index()
        self.tree_mask = self._build_tree_mask()

    def _build_parent_index(self) -> torch.Tensor:
        """mtp_engine.py:651-669."""
        parent = np.full(max(self.max_nodes, 0), -1, dtype=np.int32)
        if self.mode == "trunk":
            n = max(0, min(self.depth, self.max_nodes))
            parent[1:n] = np.arange(0, n - 1, dtype=np.int32)
        else:
            lv = _levels(self.depth, self.max_branches, self.max_nodes)
            for (ps, _), (s, n) in zip(lv[:-1], lv[1:]):
                parent[s:s + n] = ps + np.arange(n, dtype=np.int32) // self.max_branches
        return torch.from_numpy(parent)

    def _build_tree_mask(self) -> torch.Tensor:
        """mtp_engine.py:671-680: every slot sees itself; a node also sees
        each ancestor.  The parent chains are followed for all nodes at
        once, one level per step."""
        M = self.max_nodes
        mask = np.eye(M, dtype=np.float32)
        parent = self.parent.numpy().astype(np.int64)
        rows = np.arange(M)
        anc = parent.copy()
        while True:
            live = anc >= 0
            if not live.any():
                break
            mask[rows[live], anc[live]] = 1.0
            anc[live] = parent[anc[live]]
        return torch.from_numpy(mask)

    def active_node_count(self) -> int:
        """mtp_engine.py:682-685."""
        if self.mode == "trunk":
            return self.depth
        return int((self.parent >= 0).sum().item()) + 1

    def build_linear_layout(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """(depth_offsets int32 [depth + 1], branch_offsets int32
        [max_nodes]) on ``device`` (mtp_engine.py:686-713): the first node
        of each level (the last entry is ``max_nodes``; in "trunk" mode
        entry d is d - 1 and the last is ``depth``) and each node's
        position among its parent's children (0 in "trunk" mode)."""
        depth_offsets = np.zeros(self.depth + 1, dtype=np.int32)
        branch_offsets = np.zeros(max(self.max_nodes, 0), dtype=np.int32)
        if self.mode == "trunk":
            depth_offsets[1:] = np.arange(0, self.depth, dtype=np.int32)
            depth_offsets[self.depth] = self.depth
        else:
            lv = _levels(self.depth, self.max_branches, self.max_nodes)
            for d, (s, n) in enumerate(lv[1:], start=1):
                depth_offsets[d] = s
                branch_offsets[s:s + n] = np.arange(n, dtype=np.int32) % self.max_branches
            depth_offsets[self.depth] = self.max_nodes
        return (torch.from_numpy(depth_offsets).to(self.device),
                torch.from_numpy(branch_offsets).to(self.device))

    @property
    def linear_parent(self) -> torch.Tensor:
        """mtp_engine.py:715-717."""
        return self.parent.to(self.device)
