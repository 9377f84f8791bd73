"""Paged cache bookkeeping (host side): token pages, per-request page tables, the prefix cache, and the slots of
the KDA recurrent state.

The GPU caches of every MLA layer (fp8 latent + scale, rope key, index key / gate scores, pooled index keys) are
indexed by *token slot* = page id * page_size + offset; the pooled index key of pool j lives at token slot of its
first token / kpool (page_size is a multiple of kpool, so pools never straddle pages).  KDA layers keep no
per-token cache: a request owns one state slot (two buffers of the recurrent state: committed / scratch, and one
conv window).

Prefix cache: a full page is identified by a hash chained over the token ids of all pages up to and including it
(so equal hashes mean equal prefixes).  Finished requests leave their full pages in the cache (refcount 0, LRU);
a new request that starts with a cached prefix reuses those pages.  Because the KDA state is recurrent, a prefix hit
is only usable where a KDA state checkpoint exists: the engine saves the request's state at page-aligned positions
into checkpoint slots (``StateCheckpoints``), and a hit resumes from the longest prefix with both cached pages and a
checkpoint (the reference's hybrid "align-mode" prefix caching: code/kit/launcher/overlay/patch_hybrid_prefix_hit.py,
code/fork/overlay/patch_mamba_align_seed.py).
"""

from __future__ import annotations

import hashlib
from array import array
from collections import OrderedDict
from dataclasses import dataclass, field


def page_hash(prev: bytes | None, tokens: list[int]) -> bytes:
    h = hashlib.blake2b(digest_size=16)
    if prev is not None:
        h.update(prev)
    h.update(b"".join(int(t).to_bytes(4, "little", signed=False) for t in tokens))
    return h.digest()


class OutOfPages(RuntimeError):
    pass


@dataclass
class Page:
    pid: int
    ref: int = 0
    hash: bytes | None = None          # set when the page is full and registered in the prefix cache


class PageAllocator:
    """Token pages with reference counts and an LRU prefix cache of full, unreferenced pages."""

    def __init__(self, num_pages: int, page_size: int):
        self.page_size = page_size
        self.pages = [Page(i) for i in range(num_pages)]
        self.free: list[int] = list(range(num_pages - 1, -1, -1))
        self.cached: OrderedDict[bytes, int] = OrderedDict()      # hash -> pid (refcount may be > 0)
        self.stats = {"hits": 0, "queries": 0, "evictions": 0}

    @property
    def num_free(self) -> int:
        """Pages that can be handed out now (free + evictable cached pages)."""
        evictable = sum(1 for pid in self.cached.values() if self.pages[pid].ref == 0)
        return len(self.free) + evictable

    def _evict_one(self) -> int:
        for h, pid in self.cached.items():
            if self.pages[pid].ref == 0:
                del self.cached[h]
                self.pages[pid].hash = None
                self.stats["evictions"] += 1
                return pid
        raise OutOfPages("no free or evictable page")

    def alloc(self) -> int:
        pid = self.free.pop() if self.free else self._evict_one()
        p = self.pages[pid]
        p.ref = 1
        p.hash = None
        return pid

    def retain(self, pid: int) -> None:
        p = self.pages[pid]
        p.ref += 1
        if p.hash is not None and p.hash in self.cached:
            self.cached.move_to_end(p.hash)

    def release(self, pid: int) -> None:
        p = self.pages[pid]
        if p.ref <= 0:
            raise RuntimeError(f"page {pid} released twice")
        p.ref -= 1
        if p.ref == 0 and p.hash is None:
            self.free.append(pid)

    def register(self, pid: int, h: bytes) -> None:
        """Publish a full page under its prefix hash (first writer wins)."""
        if h in self.cached:
            return
        self.pages[pid].hash = h
        self.cached[h] = pid

    def lookup(self, h: bytes) -> int | None:
        self.stats["queries"] += 1
        pid = self.cached.get(h)
        if pid is not None:
            self.stats["hits"] += 1
            self.cached.move_to_end(h)
        return pid


@dataclass
class StateCheckpoint:
    slot: int                      # checkpoint slot index on the GPU
    tokens: int                    # prefix length it holds the state after
    last_used: int = 0


class StateSlots:
    """Request slots of the KDA state pool (two state buffers + one conv window each) and checkpoint slots that
    hold copies of a request's state at page-aligned prefix lengths."""

    def __init__(self, max_seqs: int, checkpoints: int = 0):
        self.free = list(range(max_seqs - 1, -1, -1))
        self.ck_free = list(range(checkpoints - 1, -1, -1))
        self.ck_by_hash: dict[bytes, StateCheckpoint] = {}
        self.clock = 0

    def alloc(self) -> int:
        if not self.free:
            raise OutOfPages("no free request slot")
        return self.free.pop()

    def release(self, slot: int) -> None:
        self.free.append(slot)

    def checkpoint_slot(self, h: bytes, tokens: int) -> StateCheckpoint | None:
        """A checkpoint slot for the prefix hash h (reusing the least recently used one when full)."""
        self.clock += 1
        if h in self.ck_by_hash:
            ck = self.ck_by_hash[h]
            ck.last_used = self.clock
            return None                                  # already stored
        if self.ck_free:
            ck = StateCheckpoint(self.ck_free.pop(), tokens, self.clock)
        elif self.ck_by_hash:
            old_h = min(self.ck_by_hash, key=lambda k: self.ck_by_hash[k].last_used)
            ck = self.ck_by_hash.pop(old_h)
            ck.tokens, ck.last_used = tokens, self.clock
        else:
            return None
        self.ck_by_hash[h] = ck
        return ck

    def find(self, h: bytes) -> StateCheckpoint | None:
        ck = self.ck_by_hash.get(h)
        if ck is not None:
            self.clock += 1
            ck.last_used = self.clock
        return ck


@dataclass
class SeqCache:
    """Cache state of one request: its page table and prefix hashes.  The page table is a compact int32 array, so
    staging it for a step is one buffer copy (16,384 pages at a 1M context) instead of a per-element conversion."""
    pages: array = field(default_factory=lambda: array("i"))
    hashes: list[bytes] = field(default_factory=list)   # hash of each full page, in order
    num_tokens: int = 0                                   # tokens with cache entries written (committed)


class KVManager:
    def __init__(self, num_pages: int, page_size: int, max_pages_per_seq: int):
        self.alloc = PageAllocator(num_pages, page_size)
        self.page_size = page_size
        self.max_pages = max_pages_per_seq

    def pages_needed(self, sc: SeqCache, upto: int) -> int:
        need = (upto + self.page_size - 1) // self.page_size
        return max(0, need - len(sc.pages))

    def can_grow(self, sc: SeqCache, upto: int) -> bool:
        return self.pages_needed(sc, upto) <= self.alloc.num_free

    def grow(self, sc: SeqCache, upto: int) -> None:
        """Make room for positions [0, upto)."""
        n = self.pages_needed(sc, upto)
        if len(sc.pages) + n > self.max_pages:
            raise OutOfPages("request exceeds max_pages_per_seq")
        for _ in range(n):
            sc.pages.append(self.alloc.alloc())

    def slot(self, sc: SeqCache, pos: int) -> int:
        return sc.pages[pos // self.page_size] * self.page_size + pos % self.page_size

    def match_prefix(self, tokens: list[int]) -> tuple[list[int], list[bytes]]:
        """Cached full pages that start ``tokens`` (longest chain), with their hashes."""
        ps = self.page_size
        pids, hashes = [], []
        prev = None
        for i in range(len(tokens) // ps):
            h = page_hash(prev, tokens[i * ps:(i + 1) * ps])
            pid = self.alloc.lookup(h)
            if pid is None:
                break
            pids.append(pid)
            hashes.append(h)
            prev = h
        return pids, hashes

    def adopt_prefix(self, sc: SeqCache, pids: list[int], hashes: list[bytes]) -> None:
        for pid in pids:
            self.alloc.retain(pid)
        sc.pages = array("i", pids)
        sc.hashes = list(hashes)
        sc.num_tokens = len(pids) * self.page_size

    def commit_tokens(self, sc: SeqCache, tokens, upto: int) -> None:
        """Positions [0, upto) are committed; publish newly full pages in the prefix cache.  `tokens` is a list or
        any object whose contiguous slices give the sequence's tokens (engine.llm.TokenView)."""
        ps = self.page_size
        sc.num_tokens = upto
        while len(sc.hashes) < upto // ps:
            i = len(sc.hashes)
            h = page_hash(sc.hashes[-1] if sc.hashes else None, tokens[i * ps:(i + 1) * ps])
            sc.hashes.append(h)
            self.alloc.register(sc.pages[i], h)

    def free(self, sc: SeqCache) -> None:
        for pid in sc.pages:
            self.alloc.release(pid)
        sc.pages = array("i")
