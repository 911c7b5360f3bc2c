"""The host page allocator of the paged KV cache (forge_paged_kv_*).
test_reference_cases follows self/test_paged_kv.hexa check by check (#1-#35);
test_random_against_model drives random operations against a direct Python
restatement of self/alloc/paged_kv.hexa (free-list stack, per-sequence
tables, alloc / release / reuse counters)."""
import numpy as np


def test_reference_cases(forge):
    a = forge.PagedKv(64, 16, 64)
    s = a.stats()
    assert (s.num_pages, a.free_count, a.used_count, a.seq_count) == (64, 64, 0, 0)           # 1-4
    p1 = a.alloc_page(1)
    assert p1 >= 0 and a.free_count == 63 and a.used_count == 1 and a.seq_pages(1) == 1       # 5-8
    p2 = a.alloc_page(1)
    assert p2 >= 0 and p2 != p1 and a.seq_pages(1) == 2                                        # 9-11
    assert a.alloc_page(2) >= 0 and a.seq_count == 2 and a.seq_pages(1) == 2 and a.seq_pages(2) == 1  # 12-15
    a.alloc_page(1)
    a.alloc_page(2)
    assert a.seq_pages(1) == 3 and a.seq_pages(2) == 2 and a.used_count == 5                   # 16-18
    t1, t2 = a.page_table(1), a.page_table(2)
    assert not set(t1) & set(t2)                                                               # 19
    free_before = a.free_count
    assert a.release_page(1, t1[0]) and a.free_count == free_before + 1 and a.seq_pages(1) == 2  # 20-22
    reuse_before = a.stats().stat_reuse
    assert a.alloc_page(1) >= 0 and a.stats().stat_reuse >= reuse_before + 1                   # 23-24
    used_before, seq2 = a.used_count, a.seq_pages(2)
    assert a.release_seq(2) and a.seq_count == 1 and a.used_count == used_before - seq2        # 25-27
    assert not a.release_page(999, 0)                                                          # 28
    b = forge.PagedKv(64, 16, 64)
    assert all(b.alloc_page(7) >= 0 for _ in range(64)) and b.free_count == 0                 # 29-30
    assert b.alloc_page(7) == -1 and b.seq_pages(7) == 64                                      # 31-32
    assert b.release_seq(7) and b.free_count == 64 and b.used_count == 0                       # 33-35


class Model:
    """self/alloc/paged_kv.hexa, restated directly."""

    def __init__(self, n):
        self.fl = list(range(n - 1, -1, -1))
        self.used = [False] * n
        self.seqs, self.tabs = [], []
        self.alloc = self.release = self.reuse = 0

    def reg(self, s):
        if s not in self.seqs:
            self.seqs.append(s)
            self.tabs.append([])

    def alloc_page(self, s):
        self.reg(s)
        if not self.fl:
            return -1
        pid = self.fl.pop()
        if not self.used[pid] and self.alloc > 0:
            self.reuse += 1
        self.used[pid] = True
        self.tabs[self.seqs.index(s)].append(pid)
        self.alloc += 1
        return pid

    def release_page(self, s, pid):
        if pid < 0 or pid >= len(self.used) or s not in self.seqs:
            return False
        t = self.tabs[self.seqs.index(s)]
        if pid not in t:
            return False
        t.remove(pid)
        self.used[pid] = False
        self.fl.append(pid)
        self.release += 1
        return True

    def release_seq(self, s):
        if s not in self.seqs:
            return False
        i = self.seqs.index(s)
        for pid in self.tabs[i]:
            self.fl.append(pid)
            self.used[pid] = False
            self.release += 1
        del self.seqs[i], self.tabs[i]
        return True


def test_random_against_model(forge):
    rng = np.random.default_rng(3)
    for trial in range(5):
        n = int(rng.integers(1, 40))
        a, m = forge.PagedKv(n, 16, 128), Model(n)
        for _ in range(400):
            op, s = int(rng.integers(0, 10)), int(rng.integers(0, 6))
            if op < 6:
                assert a.alloc_page(s) == m.alloc_page(s)
            elif op < 8:
                t = m.tabs[m.seqs.index(s)] if s in m.seqs else []
                pid = int(rng.choice(t)) if t and rng.random() < 0.8 else int(rng.integers(-2, n + 2))
                assert a.release_page(s, pid) == m.release_page(s, pid)
            else:
                assert a.release_seq(s) == m.release_seq(s)
            st = a.stats()
            assert (st.stat_alloc, st.stat_release, st.stat_reuse) == (m.alloc, m.release, m.reuse)
            assert a.free_count == len(m.fl) and a.used_count == sum(m.used) and a.seq_count == len(m.seqs)
        for s in m.seqs:
            assert a.page_table(s) == m.tabs[m.seqs.index(s)]
