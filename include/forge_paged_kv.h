/* forge_paged_kv.h — the paged KV cache: a host page allocator and
 * flash-decode over a page pool.
 *
 * The allocator keeps the contract of self/alloc/paged_kv.hexa:19-351
 * (paged_kv_new / _register_seq / _alloc_page / _release_page /
 * _release_seq / _page_table / _seq_pages / _stats): a pool of num_pages
 * pages of page_tokens tokens, a LIFO free list that hands out 0, 1, 2, ...
 * first, per-sequence page tables in allocation order, -1 when the pool is
 * exhausted, and the same alloc / release / reuse counters. It holds no
 * device memory: page ids index a caller-owned device pool.
 *
 * Device pool layout (per layer, K and V separately):
 * [num_pages][n_kv_head][page_tokens][head_dim] bf16. A sequence's row r
 * lives on page table[r / page_tokens] at row r % page_tokens. */
#ifndef FORGE_PAGED_KV_H
#define FORGE_PAGED_KV_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ForgePagedKv ForgePagedKv;

typedef struct ForgePagedKvStats {
    int32_t num_pages, page_tokens, head_dim;
    int32_t used_pages, free_pages, seq_count;
    int64_t stat_alloc, stat_release, stat_reuse;
} ForgePagedKvStats;

int  forge_paged_kv_create(int num_pages, int page_tokens, int head_dim, ForgePagedKv** out);
void forge_paged_kv_destroy(ForgePagedKv* p);
int  forge_paged_kv_free_count(const ForgePagedKv* p);
int  forge_paged_kv_used_count(const ForgePagedKv* p);
int  forge_paged_kv_seq_count(const ForgePagedKv* p);
/* Adds an empty page table for seq_id if it has none; 0. */
int  forge_paged_kv_register_seq(ForgePagedKv* p, int64_t seq_id);
/* One page appended to seq_id's table (registering it); the page id, or -1
 * when the pool is empty. */
int  forge_paged_kv_alloc_page(ForgePagedKv* p, int64_t seq_id);
/* 0, or -1 when seq_id is unknown or does not hold page_id. */
int  forge_paged_kv_release_page(ForgePagedKv* p, int64_t seq_id, int page_id);
/* Every page of seq_id back to the free list (in table order) and the
 * sequence dropped; 0, or -1 when seq_id is unknown. */
int  forge_paged_kv_release_seq(ForgePagedKv* p, int64_t seq_id);
/* Pages held by seq_id (0 when unknown); writes the first min(count, cap)
 * page ids to out. */
int  forge_paged_kv_page_table(const ForgePagedKv* p, int64_t seq_id, int32_t* out, int cap);
int  forge_paged_kv_stats(const ForgePagedKv* p, ForgePagedKvStats* out);

/* Split-K flash-decode (the same kernel and arithmetic as forge_flash_decode)
 * over page pools k_pool / v_pool of num_pages pages: block_table [B][max_pages]
 * int32 page ids (device), pos [B] the query positions (rows 0..pos[b] are
 * read, pos[b] < max_pages * page_tokens). workspace: as forge_flash_decode
 * with lmax = max_pages * page_tokens. A page id outside the pool sets the
 * error word (forge_ops_check) and the sequence's output is not written.
 * Asynchronous on stream. */
int forge_flash_decode_paged(const float* q, const uint16_t* k_pool, const uint16_t* v_pool, int num_pages,
                             const int32_t* block_table, int max_pages, int page_tokens, const int32_t* pos,
                             int B, int H, int Hkv, int hd, float* out, void* workspace, void* stream);

#ifdef __cplusplus
}
#endif
#endif
