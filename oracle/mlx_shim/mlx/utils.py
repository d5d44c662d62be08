"""``mlx.utils`` subset (test infrastructure only): parameter tree (un)flattening."""

from __future__ import annotations

from typing import Any


def tree_flatten(tree: Any, prefix: str = "", is_leaf: Any = None) -> list[tuple[str, Any]]:
    out: list[tuple[str, Any]] = []
    if isinstance(tree, dict):
        for key, value in tree.items():
            out.extend(tree_flatten(value, f"{prefix}.{key}" if prefix else str(key), is_leaf))
    elif isinstance(tree, (list, tuple)):
        for index, value in enumerate(tree):
            out.extend(tree_flatten(value, f"{prefix}.{index}" if prefix else str(index), is_leaf))
    else:
        out.append((prefix, tree))
    return out


def tree_unflatten(items: list[tuple[str, Any]]) -> Any:
    root: dict[str, Any] = {}
    for key, value in items:
        node = root
        parts = key.split(".")
        for part in parts[:-1]:
            node = node.setdefault(part, {})
        node[parts[-1]] = value
    return _listify(root)


def _listify(node: Any) -> Any:
    if not isinstance(node, dict):
        return node
    converted = {k: _listify(v) for k, v in node.items()}
    if converted and all(k.isdigit() for k in converted):
        size = max(int(k) for k in converted) + 1
        out: list[Any] = [{} for _ in range(size)]
        for k, v in converted.items():
            out[int(k)] = v
        return out
    return converted
