"""Compressed radix tree over decode-request contexts.

Requests that share a prompt prefix share one physical copy of its KV entries.
Every node owns a run of *physical positions* (indices into the shared KV pool);
a request's context is the concatenation of the positions on its root-to-node
path.

Behaviour follows the reference's ``src/tree_attention/tree.py``:

* ``KVTree.from_sequences`` (tree.py:19-50): branch on the next token, extend a
  branch while every member request agrees, allocate positions in depth-first
  first-seen order, record requests that end at a node as terminals.
* ``KVTree.synthetic`` (tree.py:52-73): a tree from parent indices, node lengths
  and the terminal node of every request; positions are allocated in node order.
* ``KVTree.extend_leaves`` (tree.py:75-88): one new position per request; a
  private childless leaf grows in place, anything else gets a new private child.
* ``storage_tokens`` (tree.py:90-92): number of physical positions.

Positions, node ids and request ids are bit-identical to the reference for the
same inputs; the scheduler's plans depend on them.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class Node:
    """One tree node: ``tokens`` are physical KV positions (reference tree.py:4-10)."""
    parent: int
    tokens: tuple[int, ...]
    children: list[int] = field(default_factory=list)
    terminal: list[int] = field(default_factory=list)
    requests: tuple[int, ...] = ()


def _empty_context_error():
    return ValueError("Every decode request needs a nonempty context")


@dataclass
class KVTree:
    """Radix tree plus each request's path of physical positions (reference tree.py:13-17)."""
    nodes: list[Node]
    paths: list[tuple[int, ...]]
    token_ids: list[int] | None = None

    @classmethod
    def from_sequences(cls, sequences):
        """Compress token sequences into a radix tree with a unique-token storage order.

        Returns a tree whose ``token_ids[p]`` is the token stored at physical
        position ``p`` and whose ``paths[r]`` lists request ``r``'s positions.
        """
        seqs = [list(s) for s in sequences]
        if not seqs or any(len(s) == 0 for s in seqs):
            raise _empty_context_error()
        tree = cls([Node(-1, ())], [None] * len(seqs), [])

        def open_node(node_id, members, depth, prefix):
            # Requests that end here become terminals; the rest are grouped by
            # their next token, in first-seen order.
            groups: dict[int, list[int]] = {}
            for r in members:
                if len(seqs[r]) == depth:
                    tree.nodes[node_id].terminal.append(r)
                    tree.paths[r] = prefix
            for r in members:
                if len(seqs[r]) > depth:
                    groups.setdefault(seqs[r][depth], []).append(r)
            return [node_id, depth, prefix, list(groups.values()), 0]

        # Depth-first expansion with an explicit stack (deeply nested trees must
        # not hit the interpreter's recursion limit).  A child is expanded fully
        # before its next sibling gets positions, which fixes the storage order.
        stack = [open_node(0, list(range(len(seqs))), 0, ())]
        while stack:
            frame = stack[-1]
            node_id, depth, prefix, groups, index = frame
            if index == len(groups):
                stack.pop()
                continue
            frame[4] = index + 1
            group = groups[index]
            lead = seqs[group[0]]
            limit = min(len(seqs[r]) for r in group)
            stop = depth + 1
            while stop < limit and all(seqs[r][stop] == lead[stop] for r in group):
                stop += 1
            first = len(tree.token_ids)
            positions = tuple(range(first, first + stop - depth))
            tree.token_ids.extend(lead[depth:stop])
            child = len(tree.nodes)
            tree.nodes.append(Node(node_id, positions, requests=tuple(group)))
            tree.nodes[node_id].children.append(child)
            stack.append(open_node(child, group, stop, prefix + positions))
        tree.nodes[0].requests = tuple(range(len(seqs)))
        return tree

    @classmethod
    def synthetic(cls, parents, lengths, terminal_nodes):
        """Tree from ``parents[i]`` (``-1`` for the root), node lengths and request terminals."""
        nodes: list[Node] = []
        next_position = 0
        for i, (parent, length) in enumerate(zip(parents, lengths)):
            valid = parent == -1 if i == 0 else 0 <= parent < i
            if not valid:
                raise ValueError("Parents must precede children")
            nodes.append(Node(parent, tuple(range(next_position, next_position + length))))
            next_position += length
            if parent >= 0:
                nodes[parent].children.append(i)
        paths = []
        for request, leaf in enumerate(terminal_nodes):
            nodes[leaf].terminal.append(request)
            chain = []
            node = leaf
            while node >= 0:
                nodes[node].requests = nodes[node].requests + (request,)
                chain.append(nodes[node].tokens)
                node = nodes[node].parent
            path = tuple(p for tokens in reversed(chain) for p in tokens)
            if not path:
                raise _empty_context_error()
            paths.append(path)
        return cls(nodes, paths)

    def extend_leaves(self, leaves, token_indices):
        """Append physical position ``token_indices[r]`` to request ``r``.

        ``leaves[r]`` is the node where request ``r`` currently ends; it is
        updated in place when a new private child has to be created.
        """
        for request, position in enumerate(token_indices):
            leaf_id = leaves[request]
            leaf = self.nodes[leaf_id]
            if leaf.requests == (request,) and not leaf.children:
                leaf.tokens = leaf.tokens + (position,)
            else:
                leaf.terminal.remove(request)
                child = len(self.nodes)
                self.nodes.append(Node(leaf_id, (position,), terminal=[request], requests=(request,)))
                leaf.children.append(child)
                leaves[request] = child
            self.paths[request] = self.paths[request] + (position,)

    @property
    def storage_tokens(self):
        """Number of physical KV positions held by the tree."""
        return sum(len(node.tokens) for node in self.nodes)
