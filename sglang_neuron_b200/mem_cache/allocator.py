"""Paged allocator and prefix cache front ends over the native runtime (C++), with pure-Python twins.

The Python twins are the executable specification the tests compare the native structures against, and
let the CPU tier run where the native module was not built.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

from .._ext import _runtime


class PyPageAllocator:
    def __init__(self, num_pages: int, page_size: int, reserved: int = 1):
        self._num_pages, self._page_size, self._reserved = num_pages, page_size, reserved
        self._free = list(range(num_pages - 1, reserved - 1, -1))
        self._staged: Dict[int, List[int]] = {}

    def available(self) -> int:
        return len(self._free)

    def staged(self) -> int:
        return sum(len(v) for v in self._staged.values())

    def num_pages(self) -> int:
        return self._num_pages

    def page_size(self) -> int:
        return self._page_size

    def alloc(self, n: int) -> List[int]:
        if n <= 0 or len(self._free) < n:
            return []
        out = self._free[-n:][::-1]
        del self._free[-n:]
        return out

    def free(self, pages: List[int]) -> None:
        for p in pages:
            if p < self._reserved or p >= self._num_pages:
                raise IndexError("freeing an invalid page id")
            self._free.append(p)

    def free_after(self, pages: List[int], epoch: int) -> None:
        self._staged.setdefault(epoch, []).extend(pages)

    def retire(self, epoch: int) -> int:
        n = 0
        for e in sorted(k for k in self._staged if k <= epoch):
            v = self._staged.pop(e)
            n += len(v)
            self.free(v)
        return n

    def reset(self) -> None:
        self._free = list(range(self._num_pages - 1, self._reserved - 1, -1))
        self._staged.clear()


def make_page_allocator(num_pages: int, page_size: int, reserved: int = 1, native: bool = True):
    if native and _runtime is not None:
        return _runtime.PageAllocator(num_pages, page_size, reserved)
    return PyPageAllocator(num_pages, page_size, reserved)


class PyRadixCache:
    """Page-granular prefix cache (reference twin of the native RadixCache)."""

    class _Node:
        __slots__ = ("key", "pages", "parent", "children", "lock", "t")

        def __init__(self, key, pages, parent):
            self.key, self.pages, self.parent = key, pages, parent
            self.children = {}
            self.lock = 0
            self.t = 0

    def __init__(self, page_size: int):
        self._ps = page_size
        self._root = self._Node((), [], None)
        self._root.lock = 1
        self._clock = 0
        self._cached = 0
        self._evictable = 0

    def page_size(self):
        return self._ps

    def cached_pages(self):
        return self._cached

    def evictable_pages(self):
        return self._evictable

    def _split(self, child, n):
        ps = self._ps
        parent = child.parent
        mid = self._Node(child.key[:n], child.pages[: n // ps], parent)
        mid.lock, mid.t = child.lock, child.t
        parent.children[child.key[:ps]] = mid
        child.key, child.pages, child.parent = child.key[n:], child.pages[n // ps:], mid
        mid.children[child.key[:ps]] = child
        return mid

    def _common(self, key, tokens, pos, limit):
        ps = self._ps
        n = 0
        while n < len(key) and pos + n + ps <= limit and tuple(key[n:n + ps]) == tuple(tokens[pos + n:pos + n + ps]):
            n += ps
        return n

    def match_prefix(self, tokens) -> Tuple[int, List[int], object]:
        tokens = tuple(tokens)
        ps = self._ps
        node, pos, pages = self._root, 0, []
        self._clock += 1
        while pos + ps <= len(tokens):
            child = node.children.get(tokens[pos:pos + ps])
            if child is None:
                break
            n = self._common(child.key, tokens, pos, len(tokens))
            if n == 0:
                break
            full = n == len(child.key)
            if not full:
                child = self._split(child, n)
            child.t = self._clock
            pages += child.pages
            pos += n
            node = child
            if not full:
                break
        return pos, pages, node

    def insert(self, tokens, pages) -> List[int]:
        tokens = tuple(tokens)
        ps = self._ps
        n_tok = (len(tokens) // ps) * ps
        node, pos, dup = self._root, 0, []
        self._clock += 1
        while pos < n_tok:
            child = node.children.get(tokens[pos:pos + ps])
            if child is None:
                new = self._Node(tokens[pos:n_tok], list(pages[pos // ps:n_tok // ps]), node)
                new.t = self._clock
                node.children[tokens[pos:pos + ps]] = new
                self._cached += len(new.pages)
                self._evictable += len(new.pages)
                return dup
            n = self._common(child.key, tokens, pos, n_tok)
            if n == 0:
                return dup
            if n < len(child.key):
                child = self._split(child, n)
            for i in range(n // ps):
                if pages[pos // ps + i] != child.pages[i]:
                    dup.append(pages[pos // ps + i])
            child.t = self._clock
            pos += n
            node = child
        return dup

    def inc_lock(self, node) -> None:
        while node is not None and node is not self._root:
            if node.lock == 0:
                self._evictable -= len(node.pages)
            node.lock += 1
            node = node.parent

    def dec_lock(self, node) -> None:
        while node is not None and node is not self._root:
            node.lock -= 1
            assert node.lock >= 0
            if node.lock == 0:
                self._evictable += len(node.pages)
            node = node.parent

    def evict(self, num_pages: int) -> List[int]:
        freed: List[int] = []
        while len(freed) < num_pages:
            leaves = []
            stack = [self._root]
            while stack:
                n = stack.pop()
                if n is not self._root and not n.children and n.lock == 0:
                    leaves.append(n)
                stack.extend(n.children.values())
            if not leaves:
                break
            v = min(leaves, key=lambda n: n.t)
            freed += v.pages
            self._cached -= len(v.pages)
            self._evictable -= len(v.pages)
            del v.parent.children[v.key[: self._ps]]
        return freed

    def reset(self) -> List[int]:
        out: List[int] = []
        stack = [self._root]
        while stack:
            n = stack.pop()
            out += n.pages
            stack.extend(n.children.values())
        self._root = self._Node((), [], None)
        self._root.lock = 1
        self._cached = self._evictable = 0
        return out


class RadixCacheHandle:
    """Uniform wrapper: the native tree hands out integer node handles, the Python twin node objects."""

    def __init__(self, page_size: int, native: bool = True):
        self.native = native and _runtime is not None
        self.tree = _runtime.RadixCache(page_size) if self.native else PyRadixCache(page_size)
        self.page_size = page_size

    def match_prefix(self, tokens):
        return self.tree.match_prefix(list(tokens))

    def insert(self, tokens, pages):
        return self.tree.insert(list(tokens), list(pages))

    def inc_lock(self, node):
        self.tree.inc_lock(node)

    def dec_lock(self, node):
        self.tree.dec_lock(node)

    def evict(self, n):
        return self.tree.evict(n)

    def evictable_pages(self):
        return self.tree.evictable_pages()

    def cached_pages(self):
        return self.tree.cached_pages()

    def reset(self):
        return self.tree.reset()
