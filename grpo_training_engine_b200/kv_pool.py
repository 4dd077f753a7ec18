"""Refcounted page pool for the paged KV cache (the KV-cache manager).

The reference allocates a fresh cache per rollout call and gives every row
of the micro-batch the SAME block table (src/triton_kernels/paged_kv.py:626-645),
so rows append into the same slots. This pool hands out distinct private
pages per sequence and lets sequences share read-only prompt pages through
reference counts (fork), with copy-on-write for a partially filled tail page
— the dense-cache semantics of the trainer's prefix expansion
(src/grpo/trainer.py:465-484), without copying full prompt pages.

Storage is one tensor per K and V:
    [num_layers, num_blocks, num_kv_heads, block_size, head_dim]
so ``pool.layer(l)`` is exactly the per-layer [num_blocks, H, bs, D] cache
the kernels take.
"""

from __future__ import annotations

from typing import Iterable, Sequence

import numpy as np
import torch


class PoolExhausted(RuntimeError):
    """Raised when an allocation asks for more pages than are free."""


class KVPagePool:
    def __init__(
        self,
        num_blocks: int,
        num_layers: int,
        num_kv_heads: int,
        block_size: int,
        head_dim: int,
        dtype: torch.dtype = torch.bfloat16,
        device: torch.device | str = "cuda",
        zero: bool = True,
    ) -> None:
        if min(num_blocks, num_layers, num_kv_heads, block_size, head_dim) <= 0:
            raise ValueError("pool dimensions must be positive.")
        self.num_blocks = int(num_blocks)
        self.num_layers = int(num_layers)
        self.num_kv_heads = int(num_kv_heads)
        self.block_size = int(block_size)
        self.head_dim = int(head_dim)
        shape = (num_layers, num_blocks, num_kv_heads, block_size, head_dim)
        alloc = torch.zeros if zero else torch.empty
        self.k = alloc(shape, dtype=dtype, device=device)
        self.v = alloc(shape, dtype=dtype, device=device)
        self._refs = np.zeros(num_blocks, dtype=np.int32)
        # LIFO free list: recently freed pages are reused first (warm in L2).
        self._free: list[int] = list(range(num_blocks - 1, -1, -1))

    # ----------------------------------------------------------- bookkeeping
    @property
    def num_free(self) -> int:
        return len(self._free)

    def refcount(self, page: int) -> int:
        return int(self._refs[page])

    def alloc(self, n: int) -> list[int]:
        """Take n free pages (refcount 1 each)."""
        if n < 0:
            raise ValueError("n must be >= 0")
        if n > len(self._free):
            raise PoolExhausted(f"requested {n} pages, {len(self._free)} free of {self.num_blocks}")
        pages = [self._free.pop() for _ in range(n)]
        self._refs[pages] = 1
        return pages

    def fork(self, pages: Iterable[int]) -> list[int]:
        """Share pages with another sequence (refcount + 1); returns the same ids."""
        pages = list(pages)
        for p in pages:
            if self._refs[p] <= 0:
                raise ValueError(f"cannot fork free page {p}")
        np.add.at(self._refs, pages, 1)
        return pages

    def free(self, pages: Iterable[int]) -> None:
        """Drop one reference per page; pages reaching zero return to the free list."""
        for p in pages:
            if self._refs[p] <= 0:
                raise ValueError(f"double free of page {p}")
            self._refs[p] -= 1
            if self._refs[p] == 0:
                self._free.append(int(p))

    def pages_for(self, num_tokens: int) -> int:
        return (int(num_tokens) + self.block_size - 1) // self.block_size

    # --------------------------------------------------------------- storage
    def layer(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.k[layer_idx], self.v[layer_idx]

    def copy_page(self, src: int, dst: int) -> None:
        """Copy one page (all layers, heads, slots) — the copy-on-write step."""
        self.k[:, dst].copy_(self.k[:, src])
        self.v[:, dst].copy_(self.v[:, src])

    def copy_pages(self, src: Sequence[int], dst: Sequence[int]) -> None:
        """Copy pages src[i] -> dst[i] (all layers) in one gather/scatter per K and V."""
        if len(src) != len(dst):
            raise ValueError("src and dst must have the same length")
        if not len(src):
            return
        si = torch.as_tensor(list(src), dtype=torch.long, device=self.k.device)
        di = torch.as_tensor(list(dst), dtype=torch.long, device=self.k.device)
        self.k[:, di] = self.k[:, si]
        self.v[:, di] = self.v[:, si]

    def make_private(self, table: list[int], index: int) -> int:
        """Copy-on-write: give `table[index]` a private copy if it is shared."""
        page = table[index]
        if self._refs[page] <= 1:
            return page
        (new,) = self.alloc(1)
        self.copy_page(page, new)
        self.free([page])
        table[index] = new
        return new

    def block_table(
        self, tables: Sequence[Sequence[int]], width: int | None = None, device=None
    ) -> torch.Tensor:
        """int32 [len(tables), width] tensor; rows are padded with page 0."""
        width = max((len(t) for t in tables), default=0) if width is None else int(width)
        arr = np.zeros((len(tables), width), dtype=np.int32)
        for i, t in enumerate(tables):
            if len(t) > width:
                raise ValueError(f"table {i} has {len(t)} pages > width {width}")
            arr[i, : len(t)] = t
        return torch.from_numpy(arr).to(self.k.device if device is None else device)

    def share_prefix(self, num_seqs: int, prefix_tokens: int, total_tokens: int) -> list[list[int]]:
        """Tables for num_seqs sequences sharing their first prefix_tokens.

        Full prefix pages are allocated once and forked; the page holding the
        prefix tail (if the prefix does not end on a page boundary) and every
        page after it are private to each sequence, since every sequence
        appends its own tokens there. Returns one page list per sequence,
        each long enough for total_tokens positions. The shared pages' data
        must be written once (through the first table) and the tail page
        copied into each private tail (see ``copy_prefix_tail``).
        """
        if num_seqs <= 0:
            return []
        full = prefix_tokens // self.block_size
        need = self.pages_for(total_tokens)
        shared = self.alloc(full)
        tables = []
        for i in range(num_seqs):
            own = self.alloc(max(need - full, 0))
            tables.append((self.fork(shared) if i > 0 else list(shared)) + own)
        return tables

    def copy_prefix_tail(self, tables: list[list[int]], prefix_tokens: int) -> None:
        """Copy the partially filled prefix page of tables[0] into the others."""
        if prefix_tokens % self.block_size == 0 or len(tables) < 2:
            return
        idx = prefix_tokens // self.block_size
        src = tables[0][idx]
        for t in tables[1:]:
            self.copy_page(src, t[idx])

    def share_prompts(
        self, groups: Sequence[int], prefix_tokens: int, total_tokens: int
    ) -> tuple[list[list[int]], list[int]]:
        """Tables for sequences whose prompts repeat: ``groups[i]`` names the prompt of row i.

        Rows of one group share their full prefix pages (``share_prefix``);
        rows of different groups share nothing. Returns one page list per row
        (in row order) and the representative row of each group (its first
        row, in order of first appearance): the prefix is written once through
        the representative's table and its partially filled tail page copied
        into the other rows' tails (``copy_prefix_tails``).
        """
        members: dict[int, list[int]] = {}
        for row, g in enumerate(groups):
            members.setdefault(int(g), []).append(row)
        tables: list[list[int]] = [[] for _ in groups]
        reps = []
        for rows in members.values():
            for row, table in zip(rows, self.share_prefix(len(rows), prefix_tokens, total_tokens)):
                tables[row] = table
            reps.append(rows[0])
        return tables, reps

    def copy_prefix_tails(self, tables: Sequence[Sequence[int]], groups: Sequence[int],
                          prefix_tokens: int) -> None:
        """Copy each group representative's partially filled prefix page into its other rows."""
        if prefix_tokens % self.block_size == 0:
            return
        idx = prefix_tokens // self.block_size
        first: dict[int, int] = {}
        src, dst = [], []
        for row, g in enumerate(groups):
            rep = first.setdefault(int(g), row)
            if rep != row:
                src.append(tables[rep][idx])
                dst.append(tables[row][idx])
        self.copy_pages(src, dst)

    @staticmethod
    def pages_needed_shared(groups: Sequence[int], prefix_tokens: int, total_tokens: int,
                            block_size: int) -> int:
        """Pages ``share_prompts`` takes: full prefix pages once per group, the rest per row."""
        full = prefix_tokens // block_size
        need = (total_tokens + block_size - 1) // block_size
        return len(set(int(g) for g in groups)) * full + len(groups) * max(need - full, 0)
