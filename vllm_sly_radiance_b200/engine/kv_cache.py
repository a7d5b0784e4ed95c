"""Paged KV-cache blocks and GDN state slots.

The hybrid model keeps two kinds of per-request cache (reference: vLLM's hybrid KV-cache manager
with the reference's group sizing, ``sly/patch_kv_groups.py``, and the mamba-style state cache,
``radiance_gdn.py:600-640``):
  * attention layers: paged K/V in blocks of ``block_size`` tokens (block 0 is reserved as the
    target of padded CUDA-graph rows);
  * GDN layers: one fixed-size state slot (conv state + SSM state) per running request
    (slot 0 reserved likewise).
Optional prefix caching hashes full blocks of prompt tokens; a hit reuses the attention blocks
and restores the GDN state snapshot taken at that block boundary.  With an offload manager
(``engine/kv_offload.py``) evicted blocks and snapshots move to host RAM / disk tiers and a hit
may continue into them.
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
                 enable_prefix_caching: bool = False, num_snapshots: int = 0,
                 snapshot_interval: int = 0):
        self.block_size = block_size
        self.blocks = BlockPool(num_blocks)
        self.slots = SlotPool(num_slots)
        self.enable_prefix_caching = enable_prefix_caching
        # GDN state snapshots: extra state slots [num_slots, num_slots + num_snapshots) holding the
        # conv + SSM state of a cached prefix at a block boundary, keyed by that prefix's hash
        # (the attention KV alone cannot resume a hybrid model: the GDN layers need their state)
        self.num_slots = num_slots
        self.num_snapshots = num_snapshots if enable_prefix_caching else 0
        self.snap_free = deque(range(num_slots, num_slots + self.num_snapshots))
        self.snap_by_hash: dict[str, int] = {}
        self.snap_lru: "OrderedDict[int, str]" = OrderedDict()
        # snapshot slots a waiting request will restore from: never recycled until the restore
        # copy is issued (or the request leaves), whatever else reserves snapshots meanwhile
        self.snap_pins: dict[int, int] = {}
        # besides the last boundary of every prompt, snapshot every `snapshot_interval` tokens
        # (rounded to blocks) so prompts that share only a leading part (a system prompt) hit
        self.snapshot_interval = (snapshot_interval // block_size * block_size
                                  if snapshot_interval else 0)
        # prefix cache: hash -> block id (LRU of unreferenced cached blocks)
        self.cached: dict[str, int] = {}
        self.block_hash: dict[int, str] = {}
        self.lru: "OrderedDict[int, None]" = OrderedDict()
        self.hits = 0
        self.queries = 0
        self.offload = None            # OffloadManager (host / disk tiers), set by the engine
        self.offload_hits = 0
        self._pending_saves: list = []

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
            if self.offload is not None:
                self._pending_saves.append((h, b))     # write-back to the host tier
        b = self.blocks.alloc()
        return b

    def flush_offload(self):
        """Enqueue the pending write-backs of evicted blocks (before anything overwrites them:
        the caller runs this before the step's forward, on the same stream)."""
        if self._pending_saves:
            self.offload.save_blocks(self._pending_saves)
            self._pending_saves = []

    def free(self, req: Request):
        self.release_restore(req)
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
        """Number of prompt tokens that can be skipped: the longest run of cached attention
        blocks whose end boundary also has a GDN state snapshot.  Sets `req.restore_snapshot`
        (the snapshot slot to copy into the request's state slot before its first step)."""
        if not self.enable_prefix_caching:
            return 0
        self.queries += 1
        if self.offload is not None:
            self.flush_offload()          # blocks evicted earlier this step become tier hits
        hs = self._hashes(req.prompt_token_ids[:-1])
        n = 0
        for h in hs:
            if h in self.cached:
                n += 1
            else:
                break
        # the run continues into the offload tiers while they hold the blocks (bounded by the
        # blocks that can be allocated for the reload)
        m = n
        if self.offload is not None:
            room = self.blocks.num_free + len(self.lru) - self.blocks_needed(req, req.num_tokens)
            while m < len(hs) and m - n < room and (hs[m] in self.cached
                                                     or self.offload.has_block(hs[m])):
                m += 1
        best, tier = 0, False
        for j in range(m, 0, -1):
            sid = self.snap_by_hash.get(hs[j - 1])
            if sid is not None:
                self.snap_lru.move_to_end(sid)
                self._pin_restore(req, sid)
                best = j
                break
            if self.offload is not None and self.num_snapshots and \
                    self.offload.has_state(hs[j - 1]) and self._can_reserve_snapshot():
                # the tier snapshot comes back into a GPU snapshot slot now (on the stream,
                # before this step's forward) and is restored from there like a resident one
                h = hs[j - 1]
                sid = self.offload.restore_state(h, lambda: self._reserve_snapshot(h))
                self._pin_restore(req, sid)
                best = j
                tier = True
                break
        if best:
            self.hits += 1
            if best > n or tier:
                self.offload_hits += 1
        return best * self.block_size

    # ---- GDN state snapshots ----
    def snapshot_boundary(self, req: Request) -> int:
        """The next token count (> computed) at which a prefill snapshots its GDN state: a
        multiple of the snapshot interval, or the last block boundary before the prompt's final
        token (0 = none left)."""
        if not self.num_snapshots:
            return 0
        last = (req.num_prompt_tokens - 1) // self.block_size * self.block_size
        c = req.num_computed_tokens
        if self.snapshot_interval:
            nxt = (c // self.snapshot_interval + 1) * self.snapshot_interval
            if nxt < last:
                return nxt
        return last if last > c else 0

    def is_snapshot_point(self, req: Request, n: int) -> bool:
        last = (req.num_prompt_tokens - 1) // self.block_size * self.block_size
        if n <= 0 or n > last:
            return False
        return n == last or (self.snapshot_interval and n % self.snapshot_interval == 0)

    def take_snapshot(self, req: Request) -> Optional[int]:
        """Reserve the snapshot slot for `req`'s prefix up to its current length when that is a
        snapshot point (None when the prefix already has one, or snapshots are off).  The
        caller copies the state into it."""
        B = req.num_computed_tokens
        if not self.num_snapshots or not self.is_snapshot_point(req, B):
            return None
        h = self._hashes(req.prompt_token_ids[:B])[-1]
        if h in self.snap_by_hash:
            return None
        return self._reserve_snapshot(h)

    def _pin_restore(self, req: Request, sid: int):
        req.restore_snapshot = sid
        self.snap_pins[sid] = self.snap_pins.get(sid, 0) + 1

    def release_restore(self, req: Request):
        """The request's pending snapshot restore is done (copy issued) or abandoned: unpin."""
        sid = req.restore_snapshot
        if sid is None:
            return
        req.restore_snapshot = None
        c = self.snap_pins.get(sid, 0) - 1
        if c > 0:
            self.snap_pins[sid] = c
        else:
            self.snap_pins.pop(sid, None)

    def _can_reserve_snapshot(self) -> bool:
        return bool(self.snap_free) or any(sid not in self.snap_pins for sid in self.snap_lru)

    def _reserve_snapshot(self, h: str) -> Optional[int]:
        """A snapshot slot for prefix hash h: a free one, else the least recently used one that
        no pending restore pins (None when every slot is pinned)."""
        if self.snap_free:
            sid = self.snap_free.popleft()
        else:
            sid = next((s for s in self.snap_lru if s not in self.snap_pins), None)
            if sid is None:
                return None
            old = self.snap_lru.pop(sid)
            self.snap_by_hash.pop(old, None)
            if self.offload is not None:
                # write-back before the new snapshot is copied into the slot
                self.offload.save_state(old, sid)
        self.snap_by_hash[h] = sid
        self.snap_lru[sid] = h
        return sid

    def adopt_prefix(self, req: Request, num_tokens: int):
        hs = self._hashes(req.prompt_token_ids[:num_tokens])
        # pin every GPU-resident block of the run first, so allocating the reloaded ones cannot
        # evict them
        got = {}
        for i, h in enumerate(hs):
            b = self.cached.get(h)
            if b is None:
                continue
            if b in self.lru:
                self.lru.pop(b)
                self.blocks.ref[b] = 1
            else:
                self.blocks.incref(b)
            got[i] = b
        loads = []
        for i, h in enumerate(hs):
            b = got.get(i)
            if b is None:
                # a block from the offload tiers: a fresh GPU block, reloaded and re-registered
                b = self._alloc_block()
                self.cached[h] = b
                self.block_hash[b] = h
                loads.append((h, b))
            req.block_ids.append(b)
        if loads:
            self.flush_offload()          # an evicted block must be saved before it is reused
            self.offload.load_blocks(loads)

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
