"""The backing pool's page allocator and token-slot expansion (CPU only).

The allocation order is part of the interface: a fresh pool hands out pages
in ascending order and reuses the most recently released page first, as the
reference allocator does (mempool/pool.py:100-125; the reference's own
checks are tests/test_core.py:27-45 and 301-316: exhaustion, double release,
page-offset bounds), and the planner fixtures' slot numbers follow from it.
"""

import types

import pytest

from cxlsparse_b200.mempool import MemoryPool, PageAllocator


def test_fresh_pool_allocates_ascending_then_reuses_last_released_first():
    pages = PageAllocator(8)
    assert pages.allocate(3) == [0, 1, 2]
    assert pages.allocate(2) == [3, 4]
    pages.release([1, 3])
    assert pages.free_pages == 5
    assert pages.allocate(1) == [3]
    assert pages.allocate(3) == [1, 5, 6]
    assert pages.allocate(0) == []
    assert pages.allocate(1) == [7]
    with pytest.raises(ValueError, match="Backing pool exhausted"):
        pages.allocate(1)
    with pytest.raises(ValueError, match="Backing pool exhausted"):
        pages.allocate(-1)


def test_release_refuses_duplicates_and_pages_not_owned():
    pages = PageAllocator(4)
    taken = pages.allocate(2)
    for bad in ([taken[0], taken[0]], [2], [9], [-1]):
        with pytest.raises(ValueError, match="Invalid page release"):
            pages.release(bad)
    assert pages.free_pages == 2  # a refused release changes nothing
    pages.release(taken)
    assert not pages.owns(taken[0]) and pages.free_pages == 4


def _pool(page_size, allocator):
    fake = types.SimpleNamespace(page_size=page_size, pages_owned=allocator)
    fake.token_slot = lambda page, offset: MemoryPool.token_slot(fake, page, offset)
    fake.token_slots = lambda pages, a, b: MemoryPool.token_slots(fake, pages, a, b)
    return fake


def test_token_slots_follow_the_page_list():
    allocator = PageAllocator(8)
    allocator.allocate(8)
    pool = _pool(64, allocator)
    pages = [5, 2, 7]
    assert pool.token_slots(pages, 10, 100) == (list(range(5 * 64 + 10, 6 * 64))
                                                + list(range(2 * 64, 2 * 64 + 36)))
    assert pool.token_slots(pages, 64, 64) == []
    assert pool.token_slots(pages, 128, 192) == list(range(7 * 64, 8 * 64))
    assert pool.token_slots(pages, 0, 192) == [pool.token_slot(pages[t // 64], t % 64)
                                               for t in range(192)]
    with pytest.raises(ValueError, match="Invalid token span"):
        pool.token_slots(pages, 0, 193)
    with pytest.raises(ValueError, match="Invalid token span"):
        pool.token_slots(pages, 5, 4)


def test_token_slot_needs_an_owned_page_and_an_offset_inside_it():
    allocator = PageAllocator(4)
    allocator.allocate(1)
    pool = _pool(16, allocator)
    assert pool.token_slot(0, 15) == 15
    for page, offset in ((1, 0), (0, 16), (0, -1), (7, 0)):
        with pytest.raises(ValueError, match="Invalid page or token offset"):
            pool.token_slot(page, offset)
    with pytest.raises(ValueError, match="Invalid page or token offset"):
        pool.token_slots([0, 1], 10, 20)  # the span reaches page 1, not owned
