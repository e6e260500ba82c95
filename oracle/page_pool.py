"""CPU restatement of the reference PagedKvPool's block-ownership model.

TEST INFRASTRUCTURE ONLY: the tests use it as the checker for the library's
page manager (inferlab_cuda_pages_*). It restates the metadata side of
PagedKvPool (worker/cpp/inferlab_runtime.cpp:649-1032); the page contents are
not modelled (the device pool holds them). Pinned by the reference's own
known-answer tests (worker/src/lib.rs:2261-2358) replayed at the page level in
tests/test_pages.py.
"""
from __future__ import annotations


class PagePoolError(RuntimeError):
    pass


class PagePool:
    def __init__(self, page_count: int, page_tokens: int, row_bytes: int, prefix_capacity: int):
        # constructor check (inferlab_runtime.cpp:661-663)
        if page_count == 0 or page_tokens == 0 or row_bytes == 0:
            raise PagePoolError("paged KV cache dimensions must be positive")
        self.page_tokens = page_tokens
        self.row_bytes = row_bytes
        self.prefix_capacity = prefix_capacity
        self.used = [0] * page_count
        self.refs = [0] * page_count
        self.live = [False] * page_count
        # free list filled with page_count - 1 .. 0, taken from the back (:668-672, :983)
        self.free = list(range(page_count - 1, -1, -1))
        self.prefixes: dict[tuple, list] = {}  # tokens -> [pages, last_used]
        self.clock = 0
        self.hits = self.misses = self.reused = 0
        self.copies = self.evictions = self.failures = 0

    # -- internals (:921-1008)
    def _page(self, pid: int) -> int:
        if pid < 0 or pid >= len(self.live) or not self.live[pid]:
            raise PagePoolError("paged KV block table contains an invalid page")
        return pid

    def _tick(self) -> int:
        self.clock += 1
        return self.clock

    def _retain(self, pid: int) -> None:
        self.refs[self._page(pid)] += 1

    def _release(self, pid: int) -> None:
        self._page(pid)
        if self.refs[pid] == 0:
            raise PagePoolError("paged KV page reference count underflow")
        self.refs[pid] -= 1
        if self.refs[pid] == 0:
            self.live[pid] = False
            self.used[pid] = 0
            self.free.append(pid)

    def _evict_oldest(self) -> None:
        if not self.prefixes:
            return
        key = min(self.prefixes, key=lambda k: self.prefixes[k][1])
        for pid in self.prefixes[key][0]:
            self._release(pid)
        del self.prefixes[key]
        self.evictions += 1

    def _allocate(self) -> int:
        while not self.free and self.prefixes:
            self._evict_oldest()
        if not self.free:
            self.failures += 1
            raise PagePoolError("paged KV cache capacity exhausted")
        pid = self.free.pop()
        self.live[pid] = True
        self.used[pid] = 0
        self.refs[pid] = 1
        return pid

    # -- public operations
    def append(self, table: list, cached_tokens: int):
        """PagedKvPool::append (:710-767) without the row write; returns the
        copy-on-write (from, to) or None. `table` is updated in place."""
        slot = cached_tokens % self.page_tokens
        if len(table) != (cached_tokens + self.page_tokens - 1) // self.page_tokens:
            raise PagePoolError("paged KV block table length is inconsistent")
        copy = None
        if slot == 0:
            pid = self._allocate()
            table.append(pid)
        else:
            if not table:
                raise PagePoolError("paged KV block table is empty for a tail row")
            pid = table[-1]
            self._page(pid)
            if self.used[pid] != slot:
                raise PagePoolError("paged KV tail occupancy is inconsistent")
            while not self.free and self.prefixes and self.refs[pid] > 1:
                self._evict_oldest()
            if self.refs[pid] > 1:
                fresh = self._allocate()
                self.used[fresh] = slot
                table[-1] = fresh
                self._release(pid)
                copy = (pid, fresh)
                self.copies += 1
                pid = fresh
        if self.refs[pid] != 1 or self.used[pid] != slot:
            raise PagePoolError("paged KV append target is not privately writable")
        self.used[pid] = slot + 1
        return copy

    def release_table(self, table: list) -> None:
        for pid in table:
            self._release(pid)
        table.clear()

    def publish_prefix(self, tokens, table: list, cached_tokens: int) -> None:
        # :805-846
        if self.prefix_capacity == 0 or len(tokens) == 0:
            return
        if len(tokens) > cached_tokens:
            raise PagePoolError("cannot publish an incomplete paged KV prefix")
        need = (len(tokens) + self.page_tokens - 1) // self.page_tokens
        if len(table) < need:
            raise PagePoolError("paged KV prefix block table is incomplete")
        pages = list(table[:need])
        key = tuple(int(t) for t in tokens)
        if key in self.prefixes:
            for pid in pages:
                self._retain(pid)
            for pid in self.prefixes[key][0]:
                self._release(pid)
            self.prefixes[key] = [pages, self._tick()]
            return
        while len(self.prefixes) >= self.prefix_capacity:
            self._evict_oldest()
        for pid in pages:
            self._retain(pid)
        self.prefixes[key] = [pages, self._tick()]

    def acquire_longest_prefix(self, tokens):
        # :679-708
        toks = tuple(int(t) for t in tokens)
        best = None
        for key in self.prefixes:
            if len(key) > len(toks) or (best is not None and len(key) <= len(best)):
                continue
            if toks[:len(key)] == key:
                best = key
        if best is None:
            self.misses += 1
            return [], 0
        for pid in self.prefixes[best][0]:
            self._retain(pid)
        self.prefixes[best][1] = self._tick()
        self.hits += 1
        self.reused += len(best)
        return list(self.prefixes[best][0]), len(best)

    def shared_pages(self, table) -> int:
        return sum(1 for pid in table if self.refs[self._page(pid)] > 1)

    def stats(self) -> dict:
        # :877-911
        r = dict.fromkeys(("allocated_pages", "used_token_slots", "live_references",
                           "maximum_refcount", "shared_pages", "physical_used_bytes",
                           "logical_referenced_bytes"), 0)
        for pid, live in enumerate(self.live):
            if not live:
                continue
            r["allocated_pages"] += 1
            r["used_token_slots"] += self.used[pid]
            r["live_references"] += self.refs[pid]
            r["maximum_refcount"] = max(r["maximum_refcount"], self.refs[pid])
            r["shared_pages"] += 1 if self.refs[pid] > 1 else 0
            r["physical_used_bytes"] += self.used[pid] * self.row_bytes
            r["logical_referenced_bytes"] += self.used[pid] * self.row_bytes * self.refs[pid]
        count = len(self.live)
        page_bytes = self.page_tokens * self.row_bytes
        r.update({
            "page_tokens": self.page_tokens, "page_count": count,
            "prefix_capacity": self.prefix_capacity, "page_bytes": page_bytes,
            "capacity_bytes": page_bytes * count,
            "free_pages": count - r["allocated_pages"],
            "allocated_token_slots": r["allocated_pages"] * self.page_tokens,
        })
        r["internal_fragmentation_bytes"] = ((r["allocated_token_slots"] - r["used_token_slots"])
                                             * self.row_bytes)
        r["bytes_saved_by_sharing"] = r["logical_referenced_bytes"] - r["physical_used_bytes"]
        r.update({"prefix_entries": len(self.prefixes), "prefix_hits": self.hits,
                  "prefix_misses": self.misses, "prefix_tokens_reused": self.reused,
                  "copy_on_write_copies": self.copies, "evictions": self.evictions,
                  "allocation_failures": self.failures})
        return r
