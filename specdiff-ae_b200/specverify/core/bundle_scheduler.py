"""Branching-ancestor bundle grouping (host logic).

Same interface and results as ``diffspec/core/bundle_scheduler.py``
(``BundleScheduler`` ``:15-289``, ``TreeDescriptorBuilder`` ``:291-392``):
leaves are bucketed by their nearest ancestor with more than one child,
buckets are visited in first-appearance order, each bucket is sorted by depth
(stable) and cut into ``bundle_size`` groups, at most ``max_bundles`` in all.

The grouping feeds :class:`specverify.runtime.bundle_verifier.FusedBundleVerifier`;
the attention kernels then score every node of a KV head in one CTA, so a
bundle's shared prefix tiles are read from memory once.  Children counts are
computed once per call here instead of once per leaf (the reference recounts
them inside ``_find_branching_ancestor``); the results are identical.
"""

from __future__ import annotations

from collections import defaultdict
from typing import Dict, List

import torch


def _children_count(parent_map: Dict[int, int]) -> Dict[int, int]:
    cnt: Dict[int, int] = defaultdict(int)
    for p in parent_map.values():
        if p >= 0:
            cnt[p] += 1
    return cnt


class BundleScheduler:
    """Group tree leaves into prefix-coherent verification bundles."""

    def __init__(self, bundle_size: int = 3, max_bundles: int = 100, device: str = "cuda"):
        self.bundle_size = bundle_size
        self.max_bundles = max_bundles
        self.device = device
        self.total_scheduled = 0
        self.total_bundles = 0
        self.avg_prefix_length = 0.0

    def schedule_bundles(self, tree_descriptor: Dict, return_tensors: bool = True) -> List[Dict]:
        leaf_ids = tree_descriptor["leaf_ids"]
        parent_map = tree_descriptor["parent_map"]
        depth_map = tree_descriptor.get("depth_map", {})
        if isinstance(leaf_ids, torch.Tensor):
            leaf_ids = leaf_ids.cpu().tolist()
        counts = _children_count(parent_map)
        buckets: Dict[int, List[int]] = {}
        for leaf in dict.fromkeys(leaf_ids):   # a repeated leaf counts once, as in the reference
            buckets.setdefault(self._branching_ancestor(leaf, parent_map, counts), []).append(leaf)
        bundles: List[Dict] = []
        for anc, leaves in buckets.items():
            if depth_map:
                leaves = sorted(leaves, key=lambda x: depth_map.get(x, 0))
            for i in range(0, len(leaves), self.bundle_size):
                group = leaves[i:i + self.bundle_size]
                prefix = self._get_path_to_ancestor(group[0], anc, parent_map) if group else []
                bundles.append({"leaves": group, "br_anc": anc, "shared_prefix": prefix,
                                "prefix_length": len(prefix), "bundle_id": len(bundles), "bucket_id": anc})
                if len(bundles) >= self.max_bundles:
                    break
            if len(bundles) >= self.max_bundles:
                break
        self.total_scheduled += len(leaf_ids)
        self.total_bundles += len(bundles)
        if bundles:
            self.avg_prefix_length = sum(b["prefix_length"] for b in bundles) / len(bundles)
        return self._convert_to_tensors(bundles) if return_tensors else bundles

    @staticmethod
    def _branching_ancestor(node: int, parent_map: Dict[int, int], counts: Dict[int, int]) -> int:
        cur = node
        while cur in parent_map:
            p = parent_map[cur]
            if p < 0:
                return cur
            if counts.get(p, 0) > 1:
                return p
            cur = p
        return 0

    def _find_branching_ancestor(self, node: int, parent_map: Dict[int, int]) -> int:
        """Nearest ancestor with more than one child (``bundle_scheduler.py:125-145``)."""
        return self._branching_ancestor(node, parent_map, _children_count(parent_map))

    def _get_path_to_ancestor(self, node: int, ancestor: int, parent_map: Dict[int, int]) -> List[int]:
        """``[ancestor, ..., node]`` (``bundle_scheduler.py:147-171``)."""
        path = []
        cur = node
        while cur != ancestor and cur in parent_map:
            path.append(cur)
            p = parent_map[cur]
            if p < 0:
                break
            cur = p
        path.append(ancestor)
        path.reverse()
        return path

    def _convert_to_tensors(self, bundles: List[Dict]) -> List[Dict]:
        out = []
        for b in bundles:
            out.append({
                "leaves": torch.tensor(b["leaves"], dtype=torch.long, device=self.device),
                "br_anc": b["br_anc"],
                "shared_prefix": torch.tensor(b["shared_prefix"], dtype=torch.long, device=self.device),
                "prefix_length": b["prefix_length"],
                "bundle_id": b["bundle_id"],
                "bucket_id": b["bucket_id"],
            })
        return out

    def create_bundle_attention_masks(self, bundles: List[Dict], max_seq_len: int) -> List[torch.Tensor]:
        """One ``[len(leaves), max_seq_len]`` int8 mask per bundle with the shared
        prefix columns set (``bundle_scheduler.py:198-242``)."""
        masks = []
        for b in bundles:
            leaves, prefix = b["leaves"], b["shared_prefix"]
            n = leaves.size(0) if isinstance(leaves, torch.Tensor) else len(leaves)
            mask = torch.zeros(n, max_seq_len, dtype=torch.int8, device=self.device)
            if isinstance(prefix, torch.Tensor) and prefix.numel() > 0:
                mask[:, prefix] = 1
            elif isinstance(prefix, list) and prefix:
                mask[:, torch.tensor(prefix, device=self.device)] = 1
            masks.append(mask)
        return masks

    def merge_bundle_logits(self, bundle_logits: List[torch.Tensor], bundles: List[Dict]) -> torch.Tensor:
        if not bundle_logits:
            return torch.empty(0, device=self.device)
        pairs = sorted(zip(bundles, bundle_logits), key=lambda x: x[0]["bundle_id"])
        return torch.cat([lg for _, lg in pairs], dim=0)

    def get_statistics(self) -> Dict:
        return {
            "total_scheduled_leaves": self.total_scheduled,
            "total_bundles_created": self.total_bundles,
            "avg_bundle_size": self.total_scheduled / self.total_bundles if self.total_bundles > 0 else 0,
            "avg_prefix_length": self.avg_prefix_length,
            "bundle_size_config": self.bundle_size,
        }

    def reset_statistics(self):
        self.total_scheduled = 0
        self.total_bundles = 0
        self.avg_prefix_length = 0.0


class TreeDescriptorBuilder:
    """Scheduler descriptors from tree representations (``bundle_scheduler.py:291-392``)."""

    @staticmethod
    def from_draft_tree(tree, final_indices: torch.Tensor = None) -> Dict:
        if final_indices is None:
            final_indices = torch.arange(tree.depth * tree.nnodes, device=tree.device)
        parent_map, depth_map = {}, {}
        idx_list = final_indices.cpu().tolist()
        for idx in idx_list:
            row, col = idx // tree.nnodes, idx % tree.nnodes
            depth_map[idx] = row
            if row > 0:
                pc = int(tree.parents_matrix[row, col].item())
                parent_map[idx] = (row - 1) * tree.nnodes + pc if pc >= 0 else -1
            else:
                parent_map[idx] = -1
        nodes = set(idx_list)
        leaves = list(nodes - (set(parent_map.values()) - {-1}))
        return {"leaf_ids": leaves, "parent_map": parent_map, "depth_map": depth_map, "all_nodes": list(nodes)}

    @staticmethod
    def from_parent_tensor(parent: torch.Tensor, num_nodes: int = None) -> Dict:
        if num_nodes is None:
            num_nodes = parent.size(0)
        plist = parent.cpu().tolist()
        parent_map = {i: (int(plist[i]) if i < len(plist) else -1) for i in range(num_nodes)}
        nodes = set(range(num_nodes))
        leaves = list(nodes - set(p for p in parent_map.values() if p >= 0))
        depth_map = {}
        for node in range(num_nodes):
            d, cur, seen = 0, node, set()
            while cur in parent_map and parent_map[cur] >= 0:
                if cur in seen:
                    break
                seen.add(cur)
                cur = parent_map[cur]
                d += 1
            depth_map[node] = d
        return {"leaf_ids": leaves, "parent_map": parent_map, "depth_map": depth_map, "all_nodes": list(nodes)}
