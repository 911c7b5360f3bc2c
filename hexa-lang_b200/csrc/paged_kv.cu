// paged_kv.cu — host page allocator of the paged KV cache (the contract of
// self/alloc/paged_kv.hexa:19-351) and the paged flash-decode entry.
//
// The reference rebuilds immutable arrays on every call; here the state is
// mutable and the operations are O(pages of the sequence): a vector free
// list used as a stack (built so pops yield 0, 1, 2, ...), a used flag per
// page, and sequence tables in registration order. The reuse counter keeps
// the reference's rule: an allocation counts as a reuse whenever any
// allocation happened before it (paged_kv.hexa:222-228).
#include <algorithm>
#include <vector>
#include "common.cuh"
#include "forge_internal.h"
#include "../../include/forge_b200.h"
#include "../../include/forge_paged_kv.h"

struct ForgePagedKv {
    int num_pages = 0, page_tokens = 0, head_dim = 0;
    std::vector<int32_t> free_list;          // stack: pop from the back
    std::vector<char> used;
    std::vector<int64_t> seq_ids;            // registration order
    std::vector<std::vector<int32_t>> tables;
    int64_t stat_alloc = 0, stat_release = 0, stat_reuse = 0;

    int find(int64_t seq) const {
        for (size_t i = 0; i < seq_ids.size(); ++i)
            if (seq_ids[i] == seq) return (int)i;
        return -1;
    }
};

extern "C" {

FORGE_API int forge_paged_kv_create(int num_pages, int page_tokens, int head_dim, ForgePagedKv** out) {
    if (!out || num_pages <= 0 || page_tokens <= 0 || head_dim <= 0)
        return forge_fail(FORGE_INVALID_ARGS, "forge_paged_kv_create: bad args");
    ForgePagedKv* p = new ForgePagedKv();
    p->num_pages = num_pages;
    p->page_tokens = page_tokens;
    p->head_dim = head_dim;
    p->free_list.resize(num_pages);
    for (int i = 0; i < num_pages; ++i) p->free_list[i] = num_pages - 1 - i;
    p->used.assign(num_pages, 0);
    *out = p;
    return 0;
}

FORGE_API void forge_paged_kv_destroy(ForgePagedKv* p) { delete p; }

FORGE_API int forge_paged_kv_free_count(const ForgePagedKv* p) { return p ? (int)p->free_list.size() : 0; }
FORGE_API int forge_paged_kv_used_count(const ForgePagedKv* p) {
    return p ? (int)std::count(p->used.begin(), p->used.end(), 1) : 0;
}
FORGE_API int forge_paged_kv_seq_count(const ForgePagedKv* p) { return p ? (int)p->seq_ids.size() : 0; }

FORGE_API int forge_paged_kv_register_seq(ForgePagedKv* p, int64_t seq) {
    if (!p) return forge_fail(FORGE_INVALID_ARGS, "forge_paged_kv_register_seq: null allocator");
    if (p->find(seq) < 0) {
        p->seq_ids.push_back(seq);
        p->tables.emplace_back();
    }
    return 0;
}

FORGE_API int forge_paged_kv_alloc_page(ForgePagedKv* p, int64_t seq) {
    if (!p) return -1;
    forge_paged_kv_register_seq(p, seq);
    if (p->free_list.empty()) return -1;
    const int32_t pid = p->free_list.back();
    p->free_list.pop_back();
    if (!p->used[pid] && p->stat_alloc > 0) ++p->stat_reuse;
    p->used[pid] = 1;
    p->tables[p->find(seq)].push_back(pid);
    ++p->stat_alloc;
    return pid;
}

FORGE_API int forge_paged_kv_release_page(ForgePagedKv* p, int64_t seq, int page_id) {
    if (!p || page_id < 0 || page_id >= p->num_pages) return -1;
    const int idx = p->find(seq);
    if (idx < 0) return -1;
    std::vector<int32_t>& t = p->tables[idx];
    auto it = std::find(t.begin(), t.end(), page_id);
    if (it == t.end()) return -1;
    t.erase(std::remove(t.begin(), t.end(), page_id), t.end());
    p->used[page_id] = 0;
    p->free_list.push_back(page_id);
    ++p->stat_release;
    return 0;
}

FORGE_API int forge_paged_kv_release_seq(ForgePagedKv* p, int64_t seq) {
    if (!p) return -1;
    const int idx = p->find(seq);
    if (idx < 0) return -1;
    for (int32_t pid : p->tables[idx]) {
        p->free_list.push_back(pid);
        p->used[pid] = 0;
        ++p->stat_release;
    }
    p->seq_ids.erase(p->seq_ids.begin() + idx);
    p->tables.erase(p->tables.begin() + idx);
    return 0;
}

FORGE_API int forge_paged_kv_page_table(const ForgePagedKv* p, int64_t seq, int32_t* out, int cap) {
    if (!p) return 0;
    const int idx = p->find(seq);
    if (idx < 0) return 0;
    const std::vector<int32_t>& t = p->tables[idx];
    for (int i = 0; out && i < cap && i < (int)t.size(); ++i) out[i] = t[i];
    return (int)t.size();
}

FORGE_API int forge_paged_kv_stats(const ForgePagedKv* p, ForgePagedKvStats* s) {
    if (!p || !s) return forge_fail(FORGE_INVALID_ARGS, "forge_paged_kv_stats: bad args");
    s->num_pages = p->num_pages;
    s->page_tokens = p->page_tokens;
    s->head_dim = p->head_dim;
    s->used_pages = forge_paged_kv_used_count(p);
    s->free_pages = forge_paged_kv_free_count(p);
    s->seq_count = forge_paged_kv_seq_count(p);
    s->stat_alloc = p->stat_alloc;
    s->stat_release = p->stat_release;
    s->stat_reuse = p->stat_reuse;
    return 0;
}

}  // extern "C"
