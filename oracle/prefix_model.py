"""TEST INFRASTRUCTURE ONLY: a pure-Python model of the paged pool's host
rules, used by tests/ (and bench.py's parity check of config 5) to check the
C++ pool (rsllm_b200/csrc/rkv_pool.cpp) decision by decision.

rsLLM has no implementation of these pieces; its plan is docs/03-HLD.md:363-376
(8.1 paged KV: per-session block table, free list, refcounted shared-prefix
blocks; 8.2 radix-tree prefix cache: token-span nodes with block ids, split on
insert, longest-prefix lookup, LRU eviction).  Parity is therefore unpinned by
the reference: this model restates the written rules of the pool, and the GPU
tests add the self-consistency checks (a gather after compaction equals the
gather before it; a branch's rows after copy-on-write equal its parent's).

Rules restated here:
  * allocation takes the lowest-numbered free page;
  * reserve(seqs, n): all-or-nothing; per sequence in order, a partially filled
    last page with refcount > 1 is copied to a fresh page first (copy-on-write),
    then new pages are taken for the remaining positions;
  * eviction takes released sequences and radix leaves in increasing
    (last_use, kind (sequence 0, node 1), id) order until `target` pages were
    freed; a node whose last child went becomes a leaf candidate;
  * compaction pairs the highest live page at or above the live count with
    the lowest free page below it, repeatedly;
  * a logical clock `tick` advances on create, fork (twice), reserve (per
    sequence), touch, insert and match, exactly as the C++ does.
"""
from __future__ import annotations

import heapq

PAGE = 64


def page_begin(t: int) -> int:
    return t // PAGE


def page_end(t: int) -> int:
    return (t + PAGE - 1) // PAGE


class PoolFull(Exception):
    pass


class OutOfRange(Exception):
    pass


class Node:
    __slots__ = ("parent", "start", "tokens", "pages", "children", "last_use", "alive")

    def __init__(self):
        self.parent = -1
        self.start = 0
        self.tokens = []
        self.pages = []
        self.children = {}
        self.last_use = 0
        self.alive = False


class Seq:
    __slots__ = ("pages", "len", "last_use", "released")

    def __init__(self):
        self.pages = []
        self.len = 0
        self.last_use = 0
        self.released = False


class PrefixModel:
    def __init__(self, n_pages: int):
        self.n_pages = n_pages
        self.ref = [0] * n_pages
        self.heap = list(range(n_pages))  # lazy min-heap of free pages
        self.n_free = n_pages
        self.seqs: dict[int, Seq] = {}
        self.next_seq = 1
        root = Node()
        root.alive = True
        self.nodes = [root]
        self.free_nodes: list[int] = []
        self.tick = 0
        self.moves: list[tuple[int, int]] = []  # (src, dst) in decision order

    # -- pages --------------------------------------------------------------
    def _alloc(self) -> int:
        while True:
            p = heapq.heappop(self.heap)
            if self.ref[p] == 0:
                self.ref[p] = 1
                self.n_free -= 1
                return p

    def _decref(self, p: int) -> bool:
        self.ref[p] -= 1
        if self.ref[p] == 0:
            heapq.heappush(self.heap, p)
            self.n_free += 1
            return True
        return False

    def _new_node(self) -> int:
        if self.free_nodes:
            i = self.free_nodes.pop()
            self.nodes[i] = Node()
        else:
            i = len(self.nodes)
            self.nodes.append(Node())
        self.nodes[i].alive = True
        return i

    # -- sequences ----------------------------------------------------------
    def create(self) -> int:
        i = self.next_seq
        self.next_seq += 1
        s = Seq()
        self.tick += 1
        s.last_use = self.tick
        self.seqs[i] = s
        return i

    def fork(self, parent: int, n: int) -> int:
        if parent not in self.seqs:
            raise OutOfRange(parent)
        p = self.seqs[parent]
        if n < 0 or n > p.len:
            raise OutOfRange(n)
        pages = p.pages[:page_end(n)]
        for x in pages:
            self.ref[x] += 1
        self.tick += 1
        p.last_use = self.tick
        i = self.next_seq
        self.next_seq += 1
        c = Seq()
        c.pages = list(pages)
        c.len = n
        self.tick += 1
        c.last_use = self.tick
        self.seqs[i] = c
        return i

    def reserve(self, seqs: list[int], ns: list[int]) -> list[int]:
        need = 0
        seen = set()
        for s, n in zip(seqs, ns):
            if s not in self.seqs:
                raise OutOfRange(s)
            if s in seen:
                raise ValueError("listed twice")
            seen.add(s)
            q = self.seqs[s]
            cow = q.len % PAGE != 0 and self.ref[q.pages[q.len // PAGE]] > 1
            need += int(cow) + page_end(q.len + n) - page_end(q.len)
        if need > self.n_free:
            raise PoolFull(need)
        slots = []
        for s, n in zip(seqs, ns):
            q = self.seqs[s]
            L = q.len
            if L % PAGE != 0 and self.ref[q.pages[L // PAGE]] > 1:
                old = q.pages[L // PAGE]
                fresh = self._alloc()
                self.moves.append((old, fresh))
                self._decref(old)
                q.pages[L // PAGE] = fresh
            for _ in range(page_end(L), page_end(L + n)):
                q.pages.append(self._alloc())
            slots.extend(q.pages[t // PAGE] * PAGE + t % PAGE for t in range(L, L + n))
            q.len = L + n
            self.tick += 1
            q.last_use = self.tick
        return slots

    def release(self, s: int) -> None:
        self.seqs[s].released = True

    def touch(self, s: int) -> None:
        self.tick += 1
        self.seqs[s].last_use = self.tick

    def free(self, s: int) -> None:
        q = self.seqs.pop(s)
        for p in q.pages:
            self._decref(p)

    # -- radix store --------------------------------------------------------
    def _split(self, nid: int, off: int) -> int:
        up_id = self._new_node()
        low = self.nodes[nid]
        up = self.nodes[up_id]
        m = low.start + off
        pb = page_begin(low.start)
        up.parent = nid
        up.start = m
        up.tokens = low.tokens[off:]
        up.children = low.children
        up.last_use = low.last_use
        for c in up.children.values():
            self.nodes[c].parent = up_id
        up.pages = low.pages[page_begin(m) - pb:]
        low.tokens = low.tokens[:off]
        low.pages = low.pages[:page_end(m) - pb]
        low.children = {up.tokens[0]: up_id}
        if m % PAGE != 0:
            self.ref[up.pages[0]] += 1
        return up_id

    def _leaf(self, parent: int, pos: int, tokens: list[int], n: int, seq: Seq, now: int) -> None:
        i = self._new_node()
        nd = self.nodes[i]
        nd.parent = parent
        nd.start = pos
        nd.tokens = list(tokens[pos:n])
        nd.pages = seq.pages[page_begin(pos):page_end(n)]
        for p in nd.pages:
            self.ref[p] += 1
        nd.last_use = now
        self.nodes[parent].children[tokens[pos]] = i

    def insert(self, tokens: list[int], seq: int) -> None:
        n = len(tokens)
        if seq not in self.seqs:
            raise OutOfRange(seq)
        s = self.seqs[seq]
        if n > s.len:
            raise OutOfRange(n)
        self.tick += 1
        now = self.tick
        cur, pos = 0, 0
        self.nodes[0].last_use = now
        while pos < n:
            child = self.nodes[cur].children.get(tokens[pos])
            if child is None:
                self._leaf(cur, pos, tokens, n, s, now)
                pos = n
                break
            c = self.nodes[child]
            span = len(c.tokens)
            j = 0
            while j < span and pos + j < n and c.tokens[j] == tokens[pos + j]:
                j += 1
            if j < span and pos + j < n:
                self._split(child, j)
            self.nodes[child].last_use = now
            cur = child
            pos += j
            if j < span:
                break
        if pos < n:
            self._leaf(cur, pos, tokens, n, s, now)
        s.last_use = now

    def match(self, tokens: list[int]) -> tuple[int, int]:
        n = len(tokens)
        self.tick += 1
        now = self.tick
        pages: list[int] = []
        cur, pos = 0, 0
        while pos < n:
            child = self.nodes[cur].children.get(tokens[pos])
            if child is None:
                break
            c = self.nodes[child]
            span = len(c.tokens)
            j = 0
            while j < span and pos + j < n and c.tokens[j] == tokens[pos + j]:
                j += 1
            pb = page_begin(c.start)
            for p in range(page_begin(pos), page_end(pos + j)):
                pg = c.pages[p - pb]
                if p < len(pages):
                    pages[p] = pg
                else:
                    pages.append(pg)
            c.last_use = now
            cur = child
            pos += j
            if j < span:
                break
        i = self.next_seq
        self.next_seq += 1
        q = Seq()
        q.pages = pages[:page_end(pos)]
        for p in q.pages:
            self.ref[p] += 1
        q.len = pos
        q.last_use = now
        self.seqs[i] = q
        return pos, i

    # -- eviction and compaction --------------------------------------------
    def evict(self, target: int) -> int:
        cand = []
        for i, q in self.seqs.items():
            if q.released:
                cand.append((q.last_use, 0, i))
        for i in range(1, len(self.nodes)):
            nd = self.nodes[i]
            if nd.alive and not nd.children:
                cand.append((nd.last_use, 1, i))
        heapq.heapify(cand)
        freed = 0
        while freed < target and cand:
            _, kind, i = heapq.heappop(cand)
            if kind == 0:
                q = self.seqs.pop(i)
                for p in q.pages:
                    freed += self._decref(p)
            else:
                nd = self.nodes[i]
                parent = nd.parent
                for p in nd.pages:
                    freed += self._decref(p)
                del self.nodes[parent].children[nd.tokens[0]]
                self.nodes[i] = Node()
                self.free_nodes.append(i)
                if parent != 0 and not self.nodes[parent].children:
                    heapq.heappush(cand, (self.nodes[parent].last_use, 1, parent))
        return freed

    def compact(self) -> list[int]:
        live = self.n_pages - self.n_free
        holes = [p for p in range(live) if self.ref[p] == 0]
        movers = [p for p in range(self.n_pages - 1, live - 1, -1) if self.ref[p] > 0]
        assert len(holes) == len(movers)
        remap = list(range(self.n_pages))
        for src, dst in zip(movers, holes):
            remap[src] = dst
            self.ref[dst] = self.ref[src]
            self.ref[src] = 0
            self.moves.append((src, dst))
        self.heap = [p for p in range(self.n_pages) if self.ref[p] == 0]
        heapq.heapify(self.heap)
        for q in self.seqs.values():
            q.pages = [remap[p] for p in q.pages]
        for nd in self.nodes:
            nd.pages = [remap[p] for p in nd.pages]
        return remap

    # -- views --------------------------------------------------------------
    def page_table(self, s: int) -> list[int]:
        return list(self.seqs[s].pages)

    def stats(self) -> dict:
        live = self.n_pages - self.n_free
        hw = 0
        for p in range(self.n_pages - 1, -1, -1):
            if self.ref[p] > 0:
                hw = p + 1
                break
        return {"free_pages": self.n_free, "live_pages": live, "sequences": len(self.seqs),
                "prefix_nodes": sum(1 for nd in self.nodes[1:] if nd.alive), "tick": self.tick, "high_water": hw}

    def take_moves(self) -> list[tuple[int, int]]:
        m, self.moves = self.moves, []
        return m
