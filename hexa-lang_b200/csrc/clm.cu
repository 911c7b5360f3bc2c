// clm.cu — host reader of the .clm int4 checkpoint format
// (stdlib/flame/clm_ckpt.hexa: save_block :47-61, load_block :63-80) and its
// conversion to the group-128 int4 layout of this library.
#include <cstdio>
#include <cstring>
#include <vector>
#include "forge_internal.h"
#include "../../include/forge_b200.h"
#include "../../include/forge_clm.h"

struct ForgeClm {
    std::vector<uint8_t> bytes;
    std::vector<ForgeClmBlock> blocks;
};

namespace {
uint32_t rd_u32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }

int clm_error(ForgeClm* c, const char* path, const char* why) {
    delete c;
    return forge_fail(FORGE_INVALID_ARGS, "forge_clm_open(%s): %s", path, why);
}

uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
}  // namespace

extern "C" {

FORGE_API int forge_clm_open(const char* path, ForgeClm** out) {
    if (!out) return forge_fail(FORGE_INVALID_ARGS, "forge_clm_open: null out");
    *out = nullptr;
    if (!path) return forge_fail(FORGE_INVALID_ARGS, "forge_clm_open: null path");
    ForgeClm* c = new ForgeClm();
    FILE* f = fopen(path, "rb");
    if (!f) return clm_error(c, path, "cannot open the file");
    uint8_t buf[1 << 16];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) c->bytes.insert(c->bytes.end(), buf, buf + n);
    fclose(f);
    const std::vector<uint8_t>& b = c->bytes;
    if (b.size() < 5 || memcmp(b.data(), "CLM\x01", 4) != 0) return clm_error(c, path, "not a .clm file (magic)");
    const int nblocks = b[4];
    size_t off = 5;
    for (int i = 0; i < nblocks; ++i) {
        if (off + 8 > b.size()) return clm_error(c, path, "truncated block header");
        ForgeClmBlock blk;
        blk.offset = (int64_t)off;
        blk.cout = rd_u32(&b[off]);
        blk.rest = rd_u32(&b[off + 4]);
        const uint64_t nel = (uint64_t)blk.cout * (uint64_t)blk.rest;
        const uint64_t need = 8 + (nel + 1) / 2 + 4 * (uint64_t)blk.cout;
        if (need > b.size() - off) return clm_error(c, path, "truncated block");
        c->blocks.push_back(blk);
        off += need;
    }
    if (off != b.size()) return clm_error(c, path, "trailing bytes after the last block");
    *out = c;
    return 0;
}

FORGE_API void forge_clm_close(ForgeClm* c) { delete c; }
FORGE_API int forge_clm_count(const ForgeClm* c) { return c ? (int)c->blocks.size() : 0; }

FORGE_API int forge_clm_block(const ForgeClm* c, int i, ForgeClmBlock* out) {
    if (!c || !out || i < 0 || i >= (int)c->blocks.size())
        return forge_fail(FORGE_INVALID_ARGS, "forge_clm_block: index %d out of range", i);
    *out = c->blocks[i];
    return 0;
}

FORGE_API int forge_clm_block_levels(const ForgeClm* c, int i, int8_t* q, float* scale) {
    ForgeClmBlock blk;
    if (forge_clm_block(c, i, &blk)) return FORGE_INVALID_ARGS;
    if (!q || !scale) return forge_fail(FORGE_INVALID_ARGS, "forge_clm_block_levels: null output");
    const uint8_t* p = c->bytes.data() + blk.offset + 8;
    const int64_t n = blk.cout * blk.rest;
    for (int64_t k = 0; k < n; k += 2) {
        const uint8_t byte = p[k / 2];
        q[k] = (int8_t)((byte & 0xF) - 8);
        if (k + 1 < n) q[k + 1] = (int8_t)(((byte >> 4) & 0xF) - 8);
    }
    memcpy(scale, p + (n + 1) / 2, 4 * (size_t)blk.cout);
    return 0;
}

FORGE_API int forge_clm_block_to_q4g128(const ForgeClm* c, int i, uint8_t* codes, uint16_t* scales) {
    ForgeClmBlock blk;
    if (forge_clm_block(c, i, &blk)) return FORGE_INVALID_ARGS;
    if (!codes || !scales) return forge_fail(FORGE_INVALID_ARGS, "forge_clm_block_to_q4g128: null output");
    if (blk.rest % 128)
        return forge_fail(FORGE_INVALID_ARGS, "forge_clm_block_to_q4g128: rest %lld is not a multiple of 128",
                          (long long)blk.rest);
    std::vector<int8_t> q((size_t)(blk.cout * blk.rest));
    std::vector<float> s((size_t)blk.cout);
    forge_clm_block_levels(c, i, q.data(), s.data());
    for (size_t k = 0; k < q.size(); ++k) {
        if (q[k] < -7)
            return forge_fail(FORGE_INVALID_ARGS, "forge_clm_block_to_q4g128: level -8 at %lld (outside [-7, 7])",
                              (long long)k);
        codes[k] = (uint8_t)(q[k] + 7);
    }
    const int64_t G = blk.rest / 128;
    for (int64_t r = 0; r < blk.cout; ++r) {
        const uint16_t sb = f32_to_bf16_rne(s[(size_t)r]);
        for (int64_t g = 0; g < G; ++g) scales[r * G + g] = sb;
    }
    return 0;
}

}  // extern "C"
