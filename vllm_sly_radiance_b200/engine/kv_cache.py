"""Paged KV-cache blocks and GDN state slots.

The hybrid model keeps two kinds of per-request cache (reference: vLLM's hybrid KV-cache manager
with the reference's group sizing, ``sly/patch_kv_groups.py``, and the mamba-style state cache,
``radiance_gdn.py:600-640``):
  * attention layers: paged K/V in blocks of ``block_size`` tokens (block 0 is reserved as the
    target of padded CUDA-graph rows);
  * GDN layers: one fixed-size state slot (conv state + SSM state) per running request
    (slot 0 reserved likewise).
Optional prefix caching hashes full blocks of prompt tokens; a hit reuses the attention blocks
and restores the GDN state snapshot taken at that block boundary.
"""
from __future__ import annotations

import hashlib
from collections import OrderedDict, deque
from typing import Optional

from .request import Request


class BlockPool:
    def __init__(self, num_blocks: int):
        if num_blocks < 2:
            raise ValueError("need at least 2 KV blocks")
        self.num_blocks = num_blocks
        self.free = deque(range(1, num_blocks))       # block 0 reserved
        self.ref = [0] * num_blocks

    @property
    def num_free(self) -> int:
        return len(self.free)

    def alloc(self) -> int:
        b = self.free.popleft()
        self.ref[b] = 1
        return b

    def incref(self, b: int):
        self.ref[b] += 1

    def release(self, b: int) -> bool:
        self.ref[b] -= 1
        if self.ref[b] == 0:
            self.free.append(b)
            return True
        return False


class SlotPool:
    def __init__(self, num_slots: int):
        self.num_slots = num_slots
        self.free = deque(range(1, num_slots))        # slot 0 reserved

    @property
    def num_free(self) -> int:
        return len(self.free)

    def alloc(self) -> int:
        return self.free.popleft()

    def release(self, s: int):
        self.free.append(s)


class KVCacheManager:
    def __init__(self, num_blocks: int, block_size: int, num_slots: int,
                 enable_prefix_caching: bool = False):
        self.block_size = block_size
        self.blocks = BlockPool(num_blocks)
        self.slots = SlotPool(num_slots)
        self.enable_prefix_caching = enable_prefix_caching
        # prefix cache: hash -> block id (LRU of unreferenced cached blocks)
        self.cached: dict[str, int] = {}
        self.block_hash: dict[int, str] = {}
        self.lru: "OrderedDict[int, None]" = OrderedDict()
        self.hits = 0
        self.queries = 0

    # ---- capacity ----
    def blocks_needed(self, req: Request, num_tokens: int) -> int:
        need = (num_tokens + self.block_size - 1) // self.block_size
        return max(0, need - len(req.block_ids))

    def can_allocate(self, req: Request, num_tokens: int) -> bool:
        extra_slot = 1 if req.state_slot is None else 0
        return (self.blocks_needed(req, num_tokens) <= self.blocks.num_free + len(self.lru)
                and extra_slot <= self.slots.num_free)

    def allocate(self, req: Request, num_tokens: int) -> bool:
        """Make room for `num_tokens` total tokens of `req`.  False when out of blocks/slots."""
        if not self.can_allocate(req, num_tokens):
            return False
        if req.state_slot is None:
            req.state_slot = self.slots.alloc()
        for _ in range(self.blocks_needed(req, num_tokens)):
            req.block_ids.append(self._alloc_block())
        return True

    def _alloc_block(self) -> int:
        if self.blocks.num_free == 0:
            # evict the least recently used cached block
            b, _ = self.lru.popitem(last=False)
            h = self.block_hash.pop(b)
            self.cached.pop(h, None)
            self.blocks.free.append(b)
        b = self.blocks.alloc()
        return b

    def free(self, req: Request):
        for b in req.block_ids:
            if self.blocks.release(b) and b in self.block_hash:
                # keep cached content around for reuse until evicted
                self.blocks.free.remove(b)
                self.lru[b] = None
        req.block_ids = []
        if req.state_slot is not None:
            self.slots.release(req.state_slot)
            req.state_slot = None

    # ---- prefix caching ----
    def _hashes(self, tokens: list[int]) -> list[str]:
        out, prev = [], ""
        for i in range(0, len(tokens) - len(tokens) % self.block_size, self.block_size):
            h = hashlib.sha1((prev + ",".join(map(str, tokens[i:i + self.block_size]))).encode()).hexdigest()
            out.append(h)
            prev = h
        return out

    def match_prefix(self, req: Request) -> int:
        """Number of prompt tokens whose attention KV is cached (a multiple of block_size).
        The GDN state at that boundary must also be available (see StateSnapshots)."""
        if not self.enable_prefix_caching:
            return 0
        self.queries += 1
        n = 0
        for h in self._hashes(req.prompt_token_ids[:-1]):
            if h in self.cached:
                n += 1
            else:
                break
        if n:
            self.hits += 1
        return n * self.block_size

    def adopt_prefix(self, req: Request, num_tokens: int):
        hs = self._hashes(req.prompt_token_ids[:num_tokens])
        for h in hs:
            b = self.cached[h]
            if b in self.lru:
                self.lru.pop(b)
                self.blocks.ref[b] = 1
            else:
                self.blocks.incref(b)
            req.block_ids.append(b)

    def register_blocks(self, req: Request):
        """After a prefill chunk: publish the full prompt blocks of `req` to the prefix cache."""
        if not self.enable_prefix_caching:
            return
        n_full = min(req.num_computed_tokens, req.num_prompt_tokens) // self.block_size
        hs = self._hashes(req.prompt_token_ids[:n_full * self.block_size])
        for i, h in enumerate(hs):
            b = req.block_ids[i]
            if h not in self.cached and b not in self.block_hash:
                self.cached[h] = b
                self.block_hash[b] = h

    @property
    def usage(self) -> float:
        used = self.blocks.num_blocks - 1 - self.blocks.num_free - len(self.lru)
        return used / max(1, self.blocks.num_blocks - 1)
