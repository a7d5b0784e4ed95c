"""KV offload tiers: host RAM and disk below the GPU prefix cache.

Reference behaviour: the reference serves with vLLM's OffloadingConnector plus 23 patches
(``kv-cache/README.md:1-60``): cached prefix blocks spill from GPU memory to a RAM tier
(/dev/shm) and a disk tier, LRU or ARC eviction, hybrid-model fixes (mamba state strides, EAGLE
groups), canonical chunks.  A hybrid GDN model cannot resume from attention KV alone, so here the
tiers hold two kinds of item, keyed by the same prefix hashes as the GPU cache:

* ``kv``: one KV block = its page in every attention layer's K and V cache;
* ``state``: one GDN state snapshot = the conv + SSM state of every GDN layer at a block
  boundary.

Items enter the host tier when the GPU cache evicts them (write-back: nothing crosses PCIe for
prefixes that stay resident).  A device kernel (``csrc/kv_copy.cu``) packs an item's segments
into a contiguous staging buffer, and one copy per item moves it to a pinned host slot.  A
prefix hit that reaches into the tiers loads the items back the same way before the step's
forward, on the same stream, so no extra synchronisation is needed.  When the host tier is full
its victim (LRU, or ARC, Megiddo & Modha 2003) is written to the disk tier (one file per item,
LRU by bytes).
"""
from __future__ import annotations

import os
from collections import OrderedDict
from typing import Optional

import numpy as np
import torch


# ---------------------------------------------------------------------------------------------
# replacement policies
# ---------------------------------------------------------------------------------------------
class LRUPolicy:
    def __init__(self, capacity: int):
        self.c = capacity
        self.od: "OrderedDict[str, None]" = OrderedDict()

    def __contains__(self, k):
        return k in self.od

    def __len__(self):
        return len(self.od)

    def hit(self, k):
        self.od.move_to_end(k)

    def insert(self, k) -> list:
        """Make k resident; returns the resident keys evicted for it."""
        out = []
        while len(self.od) >= self.c:
            out.append(self.od.popitem(last=False)[0])
        self.od[k] = None
        return out

    def remove(self, k):
        self.od.pop(k, None)


class ARCPolicy:
    """Adaptive replacement cache: recency list T1 and frequency list T2 of resident keys, ghost
    lists B1 / B2 of recently evicted ones, and the target size p of T1 adapted on ghost hits."""

    def __init__(self, capacity: int):
        self.c = capacity
        self.p = 0.0
        self.t1, self.t2, self.b1, self.b2 = (OrderedDict() for _ in range(4))

    def __contains__(self, k):
        return k in self.t1 or k in self.t2

    def __len__(self):
        return len(self.t1) + len(self.t2)

    def hit(self, k):
        if k in self.t1:
            self.t1.pop(k)
        else:
            self.t2.pop(k)
        self.t2[k] = None

    def _replace(self, in_b2: bool) -> str:
        if self.t1 and ((in_b2 and len(self.t1) == int(self.p)) or len(self.t1) > self.p):
            v = self.t1.popitem(last=False)[0]
            self.b1[v] = None
        else:
            v = self.t2.popitem(last=False)[0]
            self.b2[v] = None
        return v

    def insert(self, k) -> list:
        out = []
        if k in self.b1:
            self.p = min(self.c, self.p + max(len(self.b2) / max(len(self.b1), 1), 1))
            self.b1.pop(k)
            if len(self) >= self.c:
                out.append(self._replace(False))
            self.t2[k] = None
            return out
        if k in self.b2:
            self.p = max(0.0, self.p - max(len(self.b1) / max(len(self.b2), 1), 1))
            self.b2.pop(k)
            if len(self) >= self.c:
                out.append(self._replace(True))
            self.t2[k] = None
            return out
        l1 = len(self.t1) + len(self.b1)
        total = l1 + len(self.t2) + len(self.b2)
        if l1 >= self.c:
            if len(self.t1) < self.c:
                self.b1.popitem(last=False)
                if len(self) >= self.c:
                    out.append(self._replace(False))
            else:
                out.append(self.t1.popitem(last=False)[0])
        elif total >= self.c:
            if total >= 2 * self.c:
                self.b2.popitem(last=False)
            if len(self) >= self.c:
                out.append(self._replace(False))
        self.t1[k] = None
        return out

    def remove(self, k):
        for d in (self.t1, self.t2):
            d.pop(k, None)


def make_policy(name: str, capacity: int):
    if name == "lru":
        return LRUPolicy(capacity)
    if name == "arc":
        return ARCPolicy(capacity)
    raise ValueError(f"unknown offload policy {name!r}")


# ---------------------------------------------------------------------------------------------
# one item kind (KV blocks or GDN state slots) over its cache tensors
# ---------------------------------------------------------------------------------------------
class _Kind:
    def __init__(self, name: str, tensors: list, host_items: int, disk_dir: Optional[str],
                 disk_items: int, policy: str, device, staging_items: int):
        self.name = name
        self.tensors = tensors
        self.device = device
        self.seg_bytes = [t[0].numel() * t.element_size() for t in tensors]
        self.item_bytes = sum(self.seg_bytes)
        self.offs = []
        o = 0
        for b in self.seg_bytes:
            self.offs.append(o)
            o += b
        self.cuda = device.type == "cuda"
        self.vec = self.cuda and all(
            b % 16 == 0 and t.stride(0) * t.element_size() % 16 == 0 and t.data_ptr() % 16 == 0
            and t[0].is_contiguous() for t, b in zip(tensors, self.seg_bytes))
        if self.vec:
            self.table = torch.tensor([[t.data_ptr(), t.stride(0) * t.element_size(), b]
                                       for t, b in zip(tensors, self.seg_bytes)],
                                      dtype=torch.int64, device=device)
            self.offs_t = torch.tensor(self.offs, dtype=torch.int64, device=device)
            self.staging_items = staging_items
            self.staging = torch.empty(staging_items, self.item_bytes, dtype=torch.uint8,
                                       device=device)
        self.host_items = host_items
        self.arena = torch.empty(host_items, self.item_bytes, dtype=torch.uint8,
                                 pin_memory=self.cuda)
        self.policy = make_policy(policy, max(1, host_items))
        self.slot_of: dict[str, int] = {}
        self.free_slots = list(range(host_items - 1, -1, -1))
        self.slot_event: dict[int, torch.cuda.Event] = {}
        self.disk_dir = disk_dir
        self.disk_items = disk_items if disk_dir else 0
        self.disk: "OrderedDict[str, str]" = OrderedDict()
        self.stats = {"saved": 0, "loaded_host": 0, "loaded_disk": 0, "spilled": 0,
                      "dropped": 0}

    # ---- residency ----
    def has(self, h: str) -> bool:
        return h in self.slot_of or h in self.disk

    def _quiesce(self, slot: int):
        ev = self.slot_event.pop(slot, None)
        if ev is not None:
            ev.synchronize()

    def _evict_host(self, h: str):
        slot = self.slot_of.pop(h)
        if self.disk_items:
            self._quiesce(slot)
            while len(self.disk) >= self.disk_items:
                _, path = self.disk.popitem(last=False)
                if os.path.exists(path):
                    os.remove(path)
            path = os.path.join(self.disk_dir, f"{self.name}-{h}.bin")
            self.arena[slot].numpy().tofile(path)
            self.disk[h] = path
            self.stats["spilled"] += 1
        else:
            self.stats["dropped"] += 1
        self.free_slots.append(slot)

    def _host_slot(self, h: str) -> int:
        """A host slot for a new resident item h (evicting per the policy)."""
        for v in self.policy.insert(h):
            if v in self.slot_of:
                self._evict_host(v)
        slot = self.free_slots.pop()
        self.slot_of[h] = slot
        return slot

    def _promote(self, h: str) -> int:
        """Bring a disk item into a host slot; returns the slot."""
        path = self.disk.pop(h)
        slot = self._host_slot(h)
        self._quiesce(slot)
        data = torch.from_numpy(np.fromfile(path, dtype=np.uint8))
        self.arena[slot].copy_(data)
        os.remove(path)
        self.stats["loaded_disk"] += 1
        return slot

    # ---- transfers ----
    def save(self, items: list):
        """items: [(hash, cache index)] -> host tier (asynchronous on the current stream)."""
        items = [(h, i) for h, i in items if not self.has(h)]
        if not items or not self.host_items:
            return
        if not self.cuda:
            for h, i in items:
                slot = self._host_slot(h)
                row = self.arena[slot]
                for t, o, b in zip(self.tensors, self.offs, self.seg_bytes):
                    row[o:o + b].copy_(t[i].reshape(-1).view(torch.uint8))
                self.stats["saved"] += 1
            return
        from ..ops._ext import ext
        step = self.staging_items if self.vec else 1
        for c0 in range(0, len(items), step):
            chunk = items[c0:c0 + step]
            if self.vec:
                idx = torch.tensor([i for _, i in chunk], dtype=torch.int32).to(self.device)
                ext().segment_copy(self.table, self.offs_t, idx, self.staging, self.item_bytes,
                                   True)
            for k, (h, i) in enumerate(chunk):
                slot = self._host_slot(h)       # may spill a victim (waits for its copy)
                self._quiesce(slot)
                row = self.arena[slot]
                if self.vec:
                    row.copy_(self.staging[k], non_blocking=True)
                else:
                    for t, o, b in zip(self.tensors, self.offs, self.seg_bytes):
                        row[o:o + b].copy_(t[i].reshape(-1).view(torch.uint8), non_blocking=True)
                ev = torch.cuda.Event()
                ev.record()
                self.slot_event[slot] = ev      # the slot holds valid data once this fires
                self.stats["saved"] += 1

    def _launch_load(self, chunk: list):
        """chunk: [(host slot, cache index)], all resident: H2D + scatter on the current stream."""
        if not chunk:
            return
        if not self.cuda:
            for slot, i in chunk:
                row = self.arena[slot]
                for t, o, b in zip(self.tensors, self.offs, self.seg_bytes):
                    t[i].copy_(row[o:o + b].view(t.dtype).view(t[i].shape))
            return
        from ..ops._ext import ext
        if self.vec:
            for k, (slot, _) in enumerate(chunk):
                self.staging[k].copy_(self.arena[slot], non_blocking=True)
            idx = torch.tensor([i for _, i in chunk], dtype=torch.int32).to(self.device)
            ext().segment_copy(self.table, self.offs_t, idx, self.staging, self.item_bytes, False)
        else:
            for slot, i in chunk:
                row = self.arena[slot]
                for t, o, b in zip(self.tensors, self.offs, self.seg_bytes):
                    t[i].copy_(row[o:o + b].to(self.device, non_blocking=True)
                               .view(t.dtype).view(t[i].shape))
        ev = torch.cuda.Event()
        ev.record()
        for slot, _ in chunk:
            self.slot_event[slot] = ev          # the host slot is read until this fires

    def load(self, items: list):
        """items: [(hash, cache index)] host/disk tier -> caches (asynchronous, current stream).
        Each batch is launched before a disk item is promoted, so a promotion that evicts a
        host slot finds that slot's pending read recorded and waits for it."""
        step = self.staging_items if self.vec else 1
        chunk = []
        for h, i in items:
            if h in self.slot_of:
                self.policy.hit(h)
                slot = self.slot_of[h]
                self.stats["loaded_host"] += 1
            else:
                self._launch_load(chunk)
                chunk = []
                slot = self._promote(h)
            chunk.append((slot, i))
            if len(chunk) == step:
                self._launch_load(chunk)
                chunk = []
        self._launch_load(chunk)


    def restore_into_reserved(self, h: str, reserve) -> int:
        """Bring item h back into a cache index obtained from ``reserve()`` *after* h has been
        read out of its host slot: reserving may write back (and evict) another item, possibly
        into that very host slot.  Returns the index."""
        if h in self.slot_of:
            self.policy.hit(h)
            slot = self.slot_of[h]
            self.stats["loaded_host"] += 1
        else:
            slot = self._promote(h)
        if self.vec:
            buf = self.staging[self.staging_items - 1]
            buf.copy_(self.arena[slot], non_blocking=True)
        else:
            buf = self.arena[slot].to(self.device, copy=True)
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record()
            self.slot_event[slot] = ev
        i = reserve()
        if self.vec:
            from ..ops._ext import ext
            idx = torch.tensor([i], dtype=torch.int32).to(self.device)
            ext().segment_copy(self.table, self.offs_t, idx, buf, self.item_bytes, False)
        else:
            for t, o, b in zip(self.tensors, self.offs, self.seg_bytes):
                t[i].copy_(buf[o:o + b].view(t.dtype).view(t[i].shape))
        return i


class OffloadManager:
    """Host (pinned RAM) + optional disk tier for KV blocks and GDN state snapshots of one rank.

    ``host_bytes`` is split between the kinds by ``state_fraction``; ``disk_bytes`` likewise."""

    def __init__(self, caches, host_bytes: int, disk_dir: Optional[str] = None,
                 disk_bytes: int = 0, policy: str = "lru", state_fraction: float = 0.5,
                 staging_items: int = 8):
        dev = caches.k[0].device if caches.k else caches.conv[0].device
        kv_t = list(caches.k) + list(caches.v)
        st_t = list(caches.conv) + list(caches.ssm)
        if disk_dir:
            os.makedirs(disk_dir, exist_ok=True)

        def items(nbytes, tensors, frac):
            if not tensors:
                return 0
            per = sum(t[0].numel() * t.element_size() for t in tensors)
            return int(nbytes * frac) // per

        self.kv = _Kind("kv", kv_t, items(host_bytes, kv_t, 1 - state_fraction), disk_dir,
                        items(disk_bytes, kv_t, 1 - state_fraction), policy, dev, staging_items) \
            if kv_t else None
        self.state = _Kind("state", st_t, items(host_bytes, st_t, state_fraction), disk_dir,
                           items(disk_bytes, st_t, state_fraction), policy, dev, 2) \
            if st_t else None

    def has_block(self, h: str) -> bool:
        return self.kv is not None and self.kv.has(h)

    def has_state(self, h: str) -> bool:
        return self.state is not None and self.state.has(h)

    def save_blocks(self, items: list):
        if self.kv is not None:
            self.kv.save(items)

    def load_blocks(self, items: list):
        if self.kv is not None:
            self.kv.load(items)

    def save_state(self, h: str, slot: int):
        if self.state is not None:
            self.state.save([(h, slot)])

    def load_state(self, h: str, slot: int):
        self.state.load([(h, slot)])

    def restore_state(self, h: str, reserve) -> int:
        """Tier snapshot h -> the GPU snapshot slot that ``reserve()`` returns (see
        ``_Kind.restore_into_reserved``)."""
        return self.state.restore_into_reserved(h, reserve)

    @property
    def stats(self) -> dict:
        return {k.name: dict(k.stats, host_items=len(k.slot_of), disk_items=len(k.disk))
                for k in (self.kv, self.state) if k is not None}
