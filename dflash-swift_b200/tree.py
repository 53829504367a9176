"""Speculative tree plans: the host-side bookkeeping of a tree verify round.

A tree round verifies several drafted branches at once.  Row r of the verify block holds
one drafted token; `parents[r]` is the row it continues (-1 for the anchor, row 0).  The
plan derives what the round needs (the semantics pinned by
Tests/DFlashKitTests/SpeculativeTreeTests.swift:25-78):
  * depths: a row's distance from the anchor — its rotary position is offset + depth,
    not offset + row;
  * paths: one root-to-leaf row list per leaf;
  * row_sources: for each row, a path that contains it and its depth there;
  * attention_mask(prefix): a row sees the whole cached prefix and, in the block, only its
    own ancestors and itself (a sibling that precedes it in row order stays hidden).
After the target has scored the rows, `accepted_path` walks from the anchor into the
child whose drafted token the target named (DFlashDraftTree.acceptedPath,
Sources/DFlashKit/DFlashDraftTree.swift:122-141); the accepted rows are exactly the
`rows` argument of dflash_gdn_replay / dflash_gdn_conv_rollback (rollbackGatedDeltaTree,
DFlashSpeculativeGenerator.swift:455-456), which replay the captured inputs of those rows
in that order from the pre-round snapshot.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence, Tuple

import numpy as np


@dataclass(frozen=True)
class RowSource:
    path: int   # index into SpeculativeTreePlan.paths
    depth: int  # position of the row in that path


class SpeculativeTreePlan:
    """The shape of one tree round, from each row's parent row."""

    def __init__(self, parents: Sequence[int]):
        parents = [int(p) for p in parents]
        if not parents or parents[0] != -1:
            raise ValueError("row 0 is the anchor: parents[0] must be -1")
        for r, p in enumerate(parents[1:], start=1):
            if not 0 <= p < r:
                raise ValueError(f"row {r}: parent {p} must be an earlier row")
        self.parents = parents
        n = len(parents)
        self.children: List[List[int]] = [[] for _ in range(n)]
        for r in range(1, n):
            self.children[parents[r]].append(r)
        self.depths = [0] * n
        for r in range(1, n):
            self.depths[r] = self.depths[parents[r]] + 1
        self.paths: List[List[int]] = []
        for leaf in range(n):
            if self.children[leaf]:
                continue
            path = [leaf]
            while parents[path[-1]] >= 0:
                path.append(parents[path[-1]])
            self.paths.append(path[::-1])
        self.path_length = max(len(p) for p in self.paths)
        self.row_sources: List[RowSource] = []
        for r in range(n):
            for i, path in enumerate(self.paths):
                if r in path:
                    self.row_sources.append(RowSource(i, path.index(r)))
                    break

    @classmethod
    def chain(cls, rows: int) -> "SpeculativeTreePlan":
        """The degenerate tree of a plain chain round."""
        return cls([-1] + list(range(rows - 1)))

    @property
    def rows(self) -> int:
        return len(self.parents)

    def ancestors(self, row: int) -> List[int]:
        """The row and its ancestors, anchor first."""
        out = [row]
        while self.parents[out[-1]] >= 0:
            out.append(self.parents[out[-1]])
        return out[::-1]

    def attention_mask(self, prefix: int) -> np.ndarray:
        """bool [rows, prefix + rows]: True where a row may attend."""
        n = self.rows
        mask = np.zeros((n, prefix + n), dtype=bool)
        mask[:, :prefix] = True
        for r in range(n):
            mask[r, [prefix + a for a in self.ancestors(r)]] = True
        return mask

    def positions(self, offset: int) -> np.ndarray:
        """int32 [rows]: the rotary position of each row (offset + depth)."""
        return np.asarray([offset + d for d in self.depths], dtype=np.int32)

    def is_root_path(self, rows: Sequence[int]) -> bool:
        """Whether `rows` starts at the anchor and follows parent links."""
        rows = list(rows)
        if not rows or rows[0] != 0:
            return False
        return all(0 <= b < self.rows and self.parents[b] == a for a, b in zip(rows, rows[1:]))


def accepted_path(tokens: Sequence[int], plan: SpeculativeTreePlan,
                  target_tokens: Sequence[int]) -> Tuple[List[int], int]:
    """The rows the target agreed with, anchor first, and the target's next token after
    them.  tokens[r]: the token drafted into row r; target_tokens[r]: the target's argmax
    at row r (its continuation of row r's own path).  From the anchor, step into the
    first child (in row order) holding the token the target named, until none does."""
    if len(target_tokens) != plan.rows or len(tokens) != plan.rows:
        raise ValueError(f"{len(target_tokens)} target tokens / {len(tokens)} tokens for {plan.rows} rows")
    rows, row = [0], 0
    while True:
        nxt = next((c for c in plan.children[row] if tokens[c] == target_tokens[row]), None)
        if nxt is None:
            return rows, int(target_tokens[row])
        rows.append(nxt)
        row = nxt


def rollback_arguments(rows: Sequence[int]) -> Tuple[int, List[int]]:
    """(keep, rows) for dflash_gdn_replay / dflash_gdn_conv_rollback after a tree round."""
    rows = [int(r) for r in rows]
    return len(rows), rows
