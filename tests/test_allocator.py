"""Page allocator and page-table bookkeeping, on CPU (host-only manager).

Mirrors the reference's own allocator tests (tests/test_page_attention.cpp:4-85)
and checks every operation sequence against both the C restatement
(oracle/paged_oracle.c) and, where it was built, the reference's BlockPool
itself (oracle/_ref).
"""
import numpy as np
import pytest

from genllm_b200._lib import GkvError
from genllm_b200.paged_attention import PagedAttentionManager
from oracle.oracle import OraclePool, RefSession, ref_available


def host_mgr(capacity=None, layers=(0,), heads=8, dim=128):
    m = PagedAttentionManager(-1)
    for l in layers:
        m.init_layer(l, heads, dim)
        if capacity is not None:
            m.reserve_layer(l, capacity)
    return m


def test_block_pool_alloc_free():  # test_page_attention.cpp:4-25
    m = host_mgr(100)
    p = m.pool(0, 0)
    assert p.num_blocks() == 0 and p.num_free() == 0
    a = p.alloc()
    assert a == 0 and p.num_blocks() == 1 and p.num_free() == 0
    assert p.alloc() == 1
    p.free(a)
    assert p.num_free() == 1
    assert p.alloc() == a
    assert p.num_free() == 0


def test_block_pool_many_allocs():  # :27-35
    m = host_mgr(10)
    p = m.pool(0, 0)
    for _ in range(10):
        assert p.alloc() >= 0
    assert p.alloc() == -1


def test_block_pool_reset():  # :37-47
    m = host_mgr(10)
    p = m.pool(0, 0)
    for _ in range(3):
        p.alloc()
    p.reset()
    assert p.num_blocks() == 3 and p.num_free() == 3
    assert p.alloc() == 2  # free list refilled ascending, popped from the back


def test_page_table_append_kv():  # :49-64
    m = host_mgr(None)
    assert m.is_active(0)
    assert m.get_layer(0).num_cached == 0
    m.append_kv_pages(0, 1)
    assert m.get_layer(0).num_cached == 1
    m.append_kv_pages(0, 31)
    L = m.get_layer(0)
    assert L.num_cached == 32 and len(L.page_table) == 2


def test_page_table_multi_layer():  # :66-85
    m = PagedAttentionManager(-1)
    m.init_layer(0, 8, 128)
    m.init_layer(1, 4, 64)
    assert m.is_active(0) and m.is_active(1) and not m.is_active(2)
    m.append_kv_pages(0, 5)
    m.append_kv_pages(1, 20)
    assert m.get_layer(0).num_cached == 5 and m.get_layer(1).num_cached == 20
    m.reset()
    assert m.get_layer(0).num_cached == 0 and m.get_layer(1).page_table == []


def test_exhaustion_is_an_error_and_changes_nothing():
    # The reference breaks out of its page loop but still adds count to
    # num_cached (src/core/page_attention.cpp:155,161); here the call fails whole.
    m = host_mgr(2)
    m.append_kv_pages(0, 20)  # 2 pages
    before = m.get_layer(0)
    with pytest.raises(GkvError) as e:
        m.append_kv_pages(0, 13)  # needs a third page
    assert e.value.status == 2
    after = m.get_layer(0)
    assert after.num_cached == before.num_cached == 20
    assert after.page_table == before.page_table
    m.append_kv_pages(0, 12)  # still fits in page 2
    assert m.get_layer(0).num_cached == 32


def test_double_free_rejected():
    m = host_mgr(4)
    p = m.pool(0, 1)
    a = p.alloc()
    p.free(a)
    with pytest.raises(GkvError):
        p.free(a)
    p.free(99)  # never handed out: ignored, like the reference


def test_set_page_table_checks_ids():
    m = host_mgr(8)
    with pytest.raises(GkvError):
        m.set_page_table(0, [3], [3], 10)  # ids not handed out
    for w in (0, 1):
        for _ in range(8):
            m.pool(0, w).alloc()
    with pytest.raises(GkvError):
        m.set_page_table(0, [3], [3], 17)  # one page cannot hold 17 tokens
    m.set_page_table(0, [3, 5], [6, 1], 17)
    L = m.get_layer(0)
    assert L.num_cached == 17 and [(e.k_block_id, e.v_block_id) for e in L.page_table] == [(3, 6), (5, 1)]


def test_device_ops_refused_on_host_only_manager():
    m = host_mgr(8)
    with pytest.raises(GkvError) as e:
        m.check_device_errors(0)
    assert e.value.status == 5


def _random_ops(seed, n_ops, capacity):
    rng = np.random.default_rng(seed)
    ops = []
    for _ in range(n_ops):
        r = rng.random()
        if r < 0.45:
            ops.append(("alloc", int(rng.integers(2))))
        elif r < 0.8:
            ops.append(("free", int(rng.integers(2)), int(rng.integers(-2, capacity + 2))))
        elif r < 0.95:
            ops.append(("append", int(rng.integers(1, 40))))
        else:
            ops.append(("reset",))
    return ops


@pytest.mark.parametrize("seed", range(6))
def test_random_sequences_match_oracle_and_reference(seed):
    """Random alloc/free/append/reset sequences give the same ids, tables and
    counters as the restated BlockPool and (when built) the reference's."""
    cap = 24
    m = host_mgr(cap)
    o = OraclePool(cap)
    ref = RefSession(1, 8, 128, cap) if ref_available() else None
    freed = [set(), set()]
    for op in _random_ops(seed, 300, cap):
        if op[0] == "alloc":
            w = op[1]
            got = m.pool(0, w).alloc()
            assert got == o.alloc(w)
            if ref:
                assert got == ref.alloc(0, w)
            freed[w].discard(got)
        elif op[0] == "free":
            _, w, pid = op
            nb, _ = o.stats(w)
            if 0 <= pid < nb and pid in freed[w]:
                continue  # double free: the reference does not detect it; skip
            if 0 <= pid < nb:
                in_table = pid in (m.page_table(0)[w])
                if in_table:
                    continue  # freeing a page the table uses is a caller bug on both sides
            m.pool(0, w).free(pid)
            o.free(w, pid)
            if ref:
                ref.free(0, w, pid)
            if 0 <= pid < nb:
                freed[w].add(pid)
        elif op[0] == "append":
            cnt = op[1]
            need = sum(1 for p in range(cnt) if (o.num_cached + p) % 16 == 0)
            avail = min(cap - o.stats(w)[0] + o.stats(w)[1] for w in (0, 1))
            if need > avail:
                with pytest.raises(GkvError):
                    m.append_kv_pages(0, cnt)
                continue  # the reference's silent-corruption path is not replayed
            m.append_kv_pages(0, cnt)
            o.append_pages(cnt)
            if ref:
                ref.append_pages(0, cnt)
            for w in (0, 1):
                freed[w] -= set(int(x) for x in o.table()[w])
        else:
            m.reset()
            o.reset()
            if ref:
                ref.reset()
            nb = [o.stats(w)[0] for w in (0, 1)]
            freed = [set(range(nb[0])), set(range(nb[1]))]
        L = m.get_layer(0)
        ok, ov = o.table()
        assert L.num_cached == o.num_cached
        assert [e.k_block_id for e in L.page_table] == ok.tolist()
        assert [e.v_block_id for e in L.page_table] == ov.tolist()
        for w in (0, 1):
            assert (m.pool(0, w).num_blocks(), m.pool(0, w).num_free()) == o.stats(w)
            if ref:
                assert ref.stats(0, w) == o.stats(w)
        if ref:
            rk, rv, rn = ref.table(0)
            assert rn == o.num_cached and rk.tolist() == ok.tolist() and rv.tolist() == ov.tolist()
