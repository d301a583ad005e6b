"""Oracle: branching-ancestor bundle grouping (pure Python).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates ``BundleScheduler`` from ``diffspec/core/bundle_scheduler.py``:

* ``branching_ancestor`` (``:125-145``): walk up from a leaf; return the node
  itself if its parent is negative, the parent if that parent has more than
  one child, else continue; a node missing from the map ends at 0;
* ``path_to_ancestor`` (``:147-171``): ``[ancestor, ..., node]``;
* ``schedule`` (``:42-123``): bucket leaves by branching ancestor (bucket
  order = first appearance), sort each bucket by depth (stable), chunk into
  ``bundle_size`` groups, stop at ``max_bundles``.
"""

from __future__ import annotations

from collections import defaultdict


def branching_ancestor(node, parent_map):
    children = defaultdict(int)
    for _, p in parent_map.items():
        if p >= 0:
            children[p] += 1
    cur = node
    while cur in parent_map:
        p = parent_map[cur]
        if p < 0:
            return cur
        if children[p] > 1:
            return p
        cur = p
    return 0


def path_to_ancestor(node, ancestor, parent_map):
    path = []
    cur = node
    while cur != ancestor and cur in parent_map:
        path.append(cur)
        p = parent_map[cur]
        if p < 0:
            break
        cur = p
    path.append(ancestor)
    return path[::-1]


def schedule(leaf_ids, parent_map, depth_map, bundle_size=3, max_bundles=100):
    buckets = defaultdict(list)
    for leaf in leaf_ids:
        buckets[branching_ancestor(leaf, parent_map)].append(leaf)
    out = []
    for anc, leaves in buckets.items():
        if depth_map:
            leaves = sorted(leaves, key=lambda x: depth_map.get(x, 0))
        for i in range(0, len(leaves), bundle_size):
            grp = leaves[i:i + bundle_size]
            prefix = path_to_ancestor(grp[0], anc, parent_map) if grp else []
            out.append({"leaves": grp, "br_anc": anc, "shared_prefix": prefix,
                        "prefix_length": len(prefix), "bundle_id": len(out), "bucket_id": anc})
            if len(out) >= max_bundles:
                break
        if len(out) >= max_bundles:
            break
    return out
