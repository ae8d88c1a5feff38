"""Decoder paged K/V pool and its free list.

Same interface and allocation order as the reference's BlockManager
(speech_serving/block_manager.py:33-236): ``key_pool[l]`` / ``value_pool[l]`` are
``[num_blocks, block_size, H_kv, D]`` tensors, ``allocate_block()`` pops the END of the
free list (LIFO, :148) so block tables match the reference's block-for-block, and
exhaustion raises ``RuntimeError`` (:143-147).

B200 layout: all layers' K and V live in ONE contiguous HBM allocation
``[num_layers, 2, num_blocks, block_size, H, D]``; ``key_pool[l]`` and ``value_pool[l]``
are views of it.  A block of one layer is a contiguous ``block_size*H*D`` run — the
unit the paged attention kernel fetches with a single bulk copy.  ``block_tables()``
turns host block lists into the int32 ``[B, max_blocks]`` device table the kernels walk.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence

import torch


class BlockManager:
    def __init__(
        self,
        num_layers: int,
        num_kv_heads: int,
        head_dim: int,
        block_size: int,
        num_blocks: Optional[int] = None,
        dtype: torch.dtype = torch.float16,
        device: str = "cuda",
    ):
        dims = dict(num_layers=num_layers, num_kv_heads=num_kv_heads, head_dim=head_dim, block_size=block_size)
        bad = [k for k, v in dims.items() if v <= 0]
        if bad:
            raise ValueError("BlockManager needs positive sizes; got " + ", ".join(f"{k}={dims[k]}" for k in bad))
        self.num_layers, self.num_kv_heads, self.head_dim, self.block_size = num_layers, num_kv_heads, head_dim, \
            block_size
        self.dtype = getattr(torch, dtype) if isinstance(dtype, str) else dtype
        self.device = device
        self.num_blocks = self._auto_num_blocks() if num_blocks is None else int(num_blocks)
        if self.num_blocks <= 0:
            raise ValueError(f"BlockManager needs a positive pool size; got num_blocks={self.num_blocks}")
        self.pool = torch.zeros((num_layers, 2, self.num_blocks, block_size, num_kv_heads, head_dim),
                                dtype=self.dtype, device=device)
        self.key_pool: List[torch.Tensor] = list(self.pool[:, 0].unbind(0))
        self.value_pool: List[torch.Tensor] = list(self.pool[:, 1].unbind(0))
        self._free_list: List[int] = list(range(self.num_blocks))
        self._allocated: set = set()

    def _bytes_per_block(self) -> int:
        return self.num_layers * 2 * self.block_size * self.num_kv_heads * self.head_dim * \
            torch.tensor([], dtype=self.dtype).element_size()

    def _auto_num_blocks(self) -> int:
        """40 % of the device memory still free (reference :109-127), or 512 on CPU."""
        if not torch.cuda.is_available() or str(self.device) == "cpu":
            return 512
        free, _ = torch.cuda.mem_get_info(torch.device(self.device))
        return int(max(64, int(free * 0.40) // self._bytes_per_block()))

    def allocate_block(self) -> int:
        if not self._free_list:
            raise RuntimeError(f"decoder pool exhausted: out of physical blocks ({self.num_blocks} in use)")
        blk = self._free_list.pop()
        self._allocated.add(blk)
        return blk

    def free_blocks(self, block_ids: Sequence[int]) -> None:
        """Returns blocks to the pool; already-free ids are ignored (reference :152-166)."""
        for blk in block_ids:
            if blk in self._allocated:
                self._allocated.discard(blk)
                self._free_list.append(blk)

    @property
    def allocated_block_count(self) -> int:
        return len(self._allocated)

    @property
    def num_free_blocks(self) -> int:
        return len(self._free_list)

    def get_stats(self) -> Dict[str, Any]:
        """Occupancy counters (keys read by the scheduler and the reference's tooling:
        num_blocks, allocated_blocks, free_blocks, utilization_pct, pool_memory_mb)."""
        n, used = self.num_blocks, self.allocated_block_count
        return dict(num_blocks=n, allocated_blocks=used, free_blocks=n - used,
                    utilization_pct=round(100.0 * used / n, 2) if n else 0.0,
                    pool_memory_mb=round(self.pool.numel() * self.pool.element_size() / 2 ** 20, 2))

    def check_no_leaks(self) -> bool:
        return self.allocated_block_count == 0

    def block_tables(self, tables: Sequence[Sequence[int]], max_blocks: int, device=None,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Host block lists -> int32 [len(tables), max_blocks] (unused entries 0)."""
        t = torch.zeros((len(tables), max_blocks), dtype=torch.int32)
        for i, row in enumerate(tables):
            if len(row) > max_blocks:
                raise ValueError(f"block table of {len(row)} blocks exceeds max_blocks={max_blocks}")
            if row:
                t[i, : len(row)] = torch.tensor(list(row), dtype=torch.int32)
        dev = device if device is not None else self.device
        if out is not None:
            out.copy_(t, non_blocking=True)
            return out
        return t.to(dev)

    def __repr__(self) -> str:
        L, bs, H, D = self.num_layers, self.block_size, self.num_kv_heads, self.head_dim
        return (f"<BlockManager pool [{L}x2x{self.num_blocks}x{bs}x{H}x{D}] {self.dtype} on {self.device}: "
                f"{self.allocated_block_count} blocks in use>")
