// safetensors.cu — memory-mapped safetensors reader and the Llama-layout
// checkpoint loader (host code).
//
// The hexa runtime reaches safetensors through the RFC 025 builtins
// (self/runtime.h:1068-1082, lowered at self/codegen.hexa:7181-7186) and
// self/alloc/safetensors_mmap.hexa (tensor views over an mmap, byte
// accessor returning 0 out of range, null handle for a missing file). This
// file keeps that contract behind a C ABI: the file is mapped read-only, the
// JSON header is parsed once into views (name, dtype, shape, absolute offset,
// byte count) in header order, and tensor bytes are never copied until a
// caller asks for a converted copy. Every header field is checked (dtype
// known, shape × element size == byte count, offsets inside the file, no
// duplicate names) before the handle is returned.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "forge_internal.h"
#include "../../include/forge_safetensors.h"

struct ForgeSafetensors {
    int fd = -1;
    const uint8_t* base = nullptr;
    int64_t size = 0, header_len = 0;
    std::vector<std::string> names;
    std::vector<ForgeStTensor> views;
    std::unordered_map<std::string, int> index;
    std::unordered_map<std::string, std::string> meta;
};

namespace {

struct DtypeInfo {
    const char* name;
    int code, bytes;
};
const DtypeInfo kDtypes[] = {
    {"BOOL", FORGE_ST_BOOL, 1}, {"U8", FORGE_ST_U8, 1},         {"I8", FORGE_ST_I8, 1},
    {"I16", FORGE_ST_I16, 2},   {"U16", FORGE_ST_U16, 2},       {"F16", FORGE_ST_F16, 2},
    {"BF16", FORGE_ST_BF16, 2}, {"I32", FORGE_ST_I32, 4},       {"U32", FORGE_ST_U32, 4},
    {"F32", FORGE_ST_F32, 4},   {"F64", FORGE_ST_F64, 8},       {"I64", FORGE_ST_I64, 8},
    {"U64", FORGE_ST_U64, 8},   {"F8_E4M3", FORGE_ST_F8_E4M3, 1}, {"F8_E5M2", FORGE_ST_F8_E5M2, 1},
};
int dtype_bytes(int code) {
    for (const DtypeInfo& d : kDtypes)
        if (d.code == code) return d.bytes;
    return 0;
}

// Recursive-descent reader for the JSON subset a safetensors header uses
// (objects, arrays, strings, integers; other values are skipped).
struct JsonIn {
    const char* p;
    const char* e;
    std::string err;
    int depth = 0;

    bool fail(const char* what) {
        if (err.empty()) err = what;
        return false;
    }
    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool lit(char c) {
        ws();
        if (p < e && *p == c) {
            ++p;
            return true;
        }
        return false;
    }
    static int hexval(char c) {
        if (c >= '0' && c <= '9') return c - '0';
        if (c >= 'a' && c <= 'f') return c - 'a' + 10;
        if (c >= 'A' && c <= 'F') return c - 'A' + 10;
        return -1;
    }
    bool hex4(uint32_t& v) {
        if (e - p < 4) return fail("truncated \\u escape");
        v = 0;
        for (int i = 0; i < 4; ++i) {
            const int h = hexval(p[i]);
            if (h < 0) return fail("bad \\u escape");
            v = v * 16 + (uint32_t)h;
        }
        p += 4;
        return true;
    }
    static void utf8(std::string& s, uint32_t cp) {
        if (cp < 0x80) {
            s += (char)cp;
        } else if (cp < 0x800) {
            s += (char)(0xC0 | (cp >> 6));
            s += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            s += (char)(0xE0 | (cp >> 12));
            s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        } else {
            s += (char)(0xF0 | (cp >> 18));
            s += (char)(0x80 | ((cp >> 12) & 0x3F));
            s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        }
    }
    bool str(std::string& out) {
        out.clear();
        if (!lit('"')) return fail("expected a string");
        while (p < e) {
            const unsigned char c = (unsigned char)*p++;
            if (c == '"') return true;
            if (c < 0x20) return fail("control character in a string");
            if (c != '\\') {
                out += (char)c;
                continue;
            }
            if (p >= e) break;
            const char x = *p++;
            switch (x) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // high surrogate: a low one must follow
                        uint32_t lo;
                        if (e - p < 2 || p[0] != '\\' || p[1] != 'u') return fail("lone surrogate");
                        p += 2;
                        if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return fail("bad surrogate pair");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return fail("lone surrogate");
                    }
                    utf8(out, cp);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        return fail("unterminated string");
    }
    bool integer(int64_t& v) {
        ws();
        bool neg = false;
        if (p < e && *p == '-') {
            neg = true;
            ++p;
        }
        if (p >= e || *p < '0' || *p > '9') return fail("expected an integer");
        uint64_t u = 0;
        while (p < e && *p >= '0' && *p <= '9') {
            const uint64_t d = (uint64_t)(*p++ - '0');
            if (u > (UINT64_C(9223372036854775807) - d) / 10) return fail("integer out of range");
            u = u * 10 + d;
        }
        if (p < e && (*p == '.' || *p == 'e' || *p == 'E')) return fail("expected an integer, got a fraction");
        v = neg ? -(int64_t)u : (int64_t)u;
        return true;
    }
    bool skip() {  // any value
        ws();
        if (p >= e) return fail("truncated value");
        if (++depth > 64) return fail("nesting too deep");
        bool ok = true;
        if (*p == '"') {
            std::string s;
            ok = str(s);
        } else if (*p == '{') {
            ++p;
            if (!lit('}')) {
                do {
                    std::string k;
                    ok = str(k) && (lit(':') || fail("expected ':'")) && skip();
                } while (ok && lit(','));
                ok = ok && (lit('}') || fail("expected '}'"));
            }
        } else if (*p == '[') {
            ++p;
            if (!lit(']')) {
                do ok = skip();
                while (ok && lit(','));
                ok = ok && (lit(']') || fail("expected ']'"));
            }
        } else {
            const char* s = p;
            while (p < e && (std::isalnum((unsigned char)*p) || *p == '-' || *p == '+' || *p == '.')) ++p;
            if (p == s) ok = fail("unexpected character");
        }
        --depth;
        return ok;
    }
    bool int_array(std::vector<int64_t>& out) {
        out.clear();
        if (!lit('[')) return fail("expected an array");
        if (lit(']')) return true;
        do {
            int64_t v;
            if (!integer(v)) return false;
            out.push_back(v);
        } while (lit(','));
        return lit(']') || fail("expected ']'");
    }
};

int st_error(ForgeSafetensors* st, const char* path, const std::string& why) {
    forge_st_close(st);
    return forge_fail(FORGE_INVALID_ARGS, "forge_st_open(%s): %s", path, why.c_str());
}

// fp16 / fp64 -> fp32 and fp32 -> bf16, round to nearest even.
float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31, ex = (h >> 10) & 0x1F, man = h & 0x3FF;
    float f;
    if (ex == 0) {
        f = std::ldexp((float)man, -24);  // zero or subnormal: exact
        uint32_t u;
        memcpy(&u, &f, 4);
        u |= sign;
        memcpy(&f, &u, 4);
        return f;
    }
    const uint32_t u = ex == 31 ? (sign | 0x7F800000u | (man << 13)) : (sign | ((ex + 112) << 23) | (man << 13));
    memcpy(&f, &u, 4);
    return f;
}
uint16_t f32_bits_to_bf16(uint32_t u) {
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);  // NaN stays NaN
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return f32_bits_to_bf16(u);
}
// fp64 -> bf16 with a single rounding: fp64 -> fp32 rounded to odd (16
// spare bits, so the second rounding cannot meet a tie it did not see),
// then fp32 -> bf16 to nearest even.
uint16_t f64_to_bf16(double x) {
    if (std::isnan(x)) return std::signbit(x) ? 0xFFC0 : 0x7FC0;
    float f = (float)x;
    if (std::isfinite(x) && (double)f != x) {
        if (std::isinf(f) || std::fabs((double)f) > std::fabs(x)) f = std::nextafter(f, 0.0f);
        uint32_t u;
        memcpy(&u, &f, 4);
        u |= 1u;
        return f32_bits_to_bf16(u);
    }
    return f32_to_bf16(f);
}

template <typename T>
T load_le(const uint8_t* p) {
    T v;
    memcpy(&v, p, sizeof(T));
    return v;
}

}  // namespace

FORGE_API int forge_st_close(ForgeSafetensors* st) {
    if (!st) return 0;
    int rc = 0;
    if (st->base && munmap((void*)st->base, (size_t)st->size) != 0) rc = -1;
    if (st->fd >= 0) close(st->fd);
    delete st;
    return rc;
}

FORGE_API int forge_st_open(const char* path, ForgeSafetensors** out) {
    if (!out) return forge_fail(FORGE_INVALID_ARGS, "forge_st_open: null out");
    *out = nullptr;
    if (!path) return forge_fail(FORGE_INVALID_ARGS, "forge_st_open: null path");
    ForgeSafetensors* st = new ForgeSafetensors();
    st->fd = open(path, O_RDONLY | O_CLOEXEC);
    if (st->fd < 0) return st_error(st, path, "cannot open the file");
    struct stat sb;
    if (fstat(st->fd, &sb) != 0) return st_error(st, path, "cannot stat the file");
    st->size = (int64_t)sb.st_size;
    if (st->size < 8) return st_error(st, path, "shorter than the 8-byte header length");
    void* m = mmap(nullptr, (size_t)st->size, PROT_READ, MAP_PRIVATE, st->fd, 0);
    if (m == MAP_FAILED) return st_error(st, path, "mmap failed");
    st->base = (const uint8_t*)m;
    const uint64_t hl = load_le<uint64_t>(st->base);
    if (hl > (uint64_t)(st->size - 8)) return st_error(st, path, "header length past the end of the file");
    if (hl > 100000000u) return st_error(st, path, "header larger than the format's 100 MB limit");
    st->header_len = (int64_t)hl;
    const int64_t data0 = 8 + st->header_len;

    JsonIn js{(const char*)st->base + 8, (const char*)st->base + data0, {}};
    if (!js.lit('{')) return st_error(st, path, "header is not a JSON object");
    if (!js.lit('}')) {
        do {
            std::string name;
            if (!js.str(name) || !(js.lit(':') || js.fail("expected ':'"))) break;
            if (name == "__metadata__") {
                if (!js.lit('{')) {
                    js.fail("__metadata__ is not an object");
                    break;
                }
                if (!js.lit('}')) {
                    do {
                        std::string k, v;
                        if (!js.str(k) || !(js.lit(':') || js.fail("expected ':'")) || !js.str(v)) break;
                        st->meta[k] = v;
                    } while (js.lit(','));
                    if (!js.err.empty() || !(js.lit('}') || js.fail("expected '}'"))) break;
                }
                continue;
            }
            if (st->index.count(name)) {
                js.fail("duplicate tensor name");
                break;
            }
            ForgeStTensor v{};
            v.dtype = -1;
            std::vector<int64_t> shape, offs;
            bool have_shape = false, have_offs = false;
            if (!js.lit('{')) {
                js.fail("tensor entry is not an object");
                break;
            }
            if (!js.lit('}')) {
                do {
                    std::string k;
                    if (!js.str(k) || !(js.lit(':') || js.fail("expected ':'"))) break;
                    if (k == "dtype") {
                        std::string dt;
                        if (!js.str(dt)) break;
                        for (const DtypeInfo& d : kDtypes)
                            if (dt == d.name) v.dtype = d.code;
                        if (v.dtype < 0) {
                            js.err = "tensor " + name + ": unknown dtype " + dt;
                            break;
                        }
                    } else if (k == "shape") {
                        if (!js.int_array(shape)) break;
                        have_shape = true;
                    } else if (k == "data_offsets") {
                        if (!js.int_array(offs)) break;
                        have_offs = true;
                    } else if (!js.skip()) {
                        break;
                    }
                } while (js.lit(','));
                if (!js.err.empty() || !(js.lit('}') || js.fail("expected '}'"))) break;
            }
            if (v.dtype < 0 || !have_shape || !have_offs) {
                js.err = "tensor " + name + ": needs dtype, shape and data_offsets";
                break;
            }
            if ((int)shape.size() > FORGE_ST_MAX_DIMS || offs.size() != 2) {
                js.err = "tensor " + name + ": more than 8 dimensions or data_offsets not a pair";
                break;
            }
            int64_t numel = 1;
            bool bad = false;
            for (size_t i = 0; i < shape.size(); ++i) {
                if (shape[i] < 0 || (shape[i] && numel > INT64_MAX / 8 / shape[i])) bad = true;
                else numel *= shape[i];
                v.shape[i] = shape[i];
            }
            v.ndim = (int)shape.size();
            if (bad) {
                js.err = "tensor " + name + ": bad shape";
                break;
            }
            if (offs[0] < 0 || offs[1] < offs[0] || offs[1] > st->size - data0) {
                js.err = "tensor " + name + ": data_offsets outside the data region";
                break;
            }
            v.nbytes = offs[1] - offs[0];
            if (v.nbytes != numel * dtype_bytes(v.dtype)) {
                js.err = "tensor " + name + ": byte count does not match dtype and shape";
                break;
            }
            v.offset = data0 + offs[0];
            v.data = st->base + v.offset;
            st->index[name] = (int)st->names.size();
            st->names.push_back(name);
            st->views.push_back(v);
        } while (js.lit(','));
        if (js.err.empty() && !js.lit('}')) js.fail("expected '}' at the end of the header");
    }
    if (!js.err.empty()) return st_error(st, path, js.err);
    js.ws();  // the header may be padded with spaces
    if (js.p != js.e) return st_error(st, path, "trailing bytes after the header object");
    for (size_t i = 0; i < st->views.size(); ++i) st->views[i].name = st->names[i].c_str();
    *out = st;
    return 0;
}

FORGE_API const char* forge_st_header(const ForgeSafetensors* st, int64_t* len) {
    if (len) *len = st ? st->header_len : 0;
    return st ? (const char*)st->base + 8 : nullptr;
}
FORGE_API int64_t forge_st_data_offset(const ForgeSafetensors* st) { return st ? 8 + st->header_len : -1; }
FORGE_API int64_t forge_st_size(const ForgeSafetensors* st) { return st ? st->size : -1; }
FORGE_API int forge_st_count(const ForgeSafetensors* st) { return st ? (int)st->views.size() : 0; }
FORGE_API int64_t forge_st_total_bytes(const ForgeSafetensors* st) {
    int64_t s = 0;
    if (st)
        for (const ForgeStTensor& v : st->views) s += v.nbytes;
    return s;
}
FORGE_API int forge_st_tensor_at(const ForgeSafetensors* st, int i, ForgeStTensor* out) {
    if (!st || !out || i < 0 || i >= (int)st->views.size())
        return forge_fail(FORGE_INVALID_ARGS, "forge_st_tensor_at: index %d out of range", i);
    *out = st->views[i];
    return 0;
}
FORGE_API int forge_st_find(const ForgeSafetensors* st, const char* name, ForgeStTensor* out) {
    if (out) *out = ForgeStTensor{};
    if (!st || !name || !out) return forge_fail(FORGE_INVALID_ARGS, "forge_st_find: bad args");
    auto it = st->index.find(name);
    if (it == st->index.end()) return FORGE_ST_NOT_FOUND;
    *out = st->views[it->second];
    return 0;
}
FORGE_API const char* forge_st_metadata(const ForgeSafetensors* st, const char* key) {
    if (!st || !key) return nullptr;
    auto it = st->meta.find(key);
    return it == st->meta.end() ? nullptr : it->second.c_str();
}
FORGE_API int forge_st_view_u8(const ForgeStTensor* v, int64_t i) {
    if (!v || !v->data || i < 0 || i >= v->nbytes) return 0;
    return ((const uint8_t*)v->data)[i];
}

namespace {
bool in_file(const ForgeSafetensors* st, int64_t off, int64_t n, int64_t esz) {
    return st && off >= 0 && n >= 0 && n <= (INT64_MAX - off) / esz && off + n * esz <= st->size;
}
}  // namespace

FORGE_API int64_t forge_st_read_bytes(const ForgeSafetensors* st, int64_t off, int64_t n, void* out) {
    if (!in_file(st, off, n, 1) || (n && !out))
        return forge_fail(FORGE_INVALID_ARGS, "forge_st_read_bytes: [%lld, +%lld) outside the file", (long long)off,
                          (long long)n);
    if (n) memcpy(out, st->base + off, (size_t)n);
    return n;
}
FORGE_API int64_t forge_st_read_f32(const ForgeSafetensors* st, int64_t off, int64_t n, float* out) {
    if (!in_file(st, off, n, 4) || (n && !out))
        return forge_fail(FORGE_INVALID_ARGS, "forge_st_read_f32: %lld floats at %lld outside the file", (long long)n,
                          (long long)off);
    if (n) memcpy(out, st->base + off, (size_t)n * 4);
    return n;
}
FORGE_API int64_t forge_st_read_bf16_to_f32(const ForgeSafetensors* st, int64_t off, int64_t n, float* out) {
    if (!in_file(st, off, n, 2) || (n && !out))
        return forge_fail(FORGE_INVALID_ARGS, "forge_st_read_bf16_to_f32: %lld values at %lld outside the file",
                          (long long)n, (long long)off);
    for (int64_t i = 0; i < n; ++i) {
        const uint32_t u = (uint32_t)load_le<uint16_t>(st->base + off + 2 * i) << 16;
        memcpy(out + i, &u, 4);
    }
    return n;
}

FORGE_API int forge_st_tensor_to_bf16(const ForgeStTensor* v, uint16_t* out, int64_t n) {
    if (!v || !v->data || !out) return forge_fail(FORGE_INVALID_ARGS, "forge_st_tensor_to_bf16: bad args");
    const int esz = dtype_bytes(v->dtype);
    if (!esz || n * esz != v->nbytes)
        return forge_fail(FORGE_INVALID_ARGS, "forge_st_tensor_to_bf16: %s holds %lld bytes, not %lld values",
                          v->name ? v->name : "?", (long long)v->nbytes, (long long)n);
    const uint8_t* p = (const uint8_t*)v->data;
    switch (v->dtype) {
        case FORGE_ST_BF16: memcpy(out, p, (size_t)n * 2); break;
        case FORGE_ST_F32:
            for (int64_t i = 0; i < n; ++i) out[i] = f32_bits_to_bf16(load_le<uint32_t>(p + 4 * i));
            break;
        case FORGE_ST_F16:
            for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16(f16_to_f32(load_le<uint16_t>(p + 2 * i)));
            break;
        case FORGE_ST_F64:
            for (int64_t i = 0; i < n; ++i) out[i] = f64_to_bf16(load_le<double>(p + 8 * i));
            break;
        default:
            return forge_fail(FORGE_INVALID_ARGS, "forge_st_tensor_to_bf16: %s is not a floating-point tensor",
                              v->name ? v->name : "?");
    }
    return 0;
}

FORGE_API int forge_st_tensor_to_f32(const ForgeStTensor* v, float* out, int64_t n) {
    if (!v || !v->data || !out) return forge_fail(FORGE_INVALID_ARGS, "forge_st_tensor_to_f32: bad args");
    const int esz = dtype_bytes(v->dtype);
    if (!esz || n * esz != v->nbytes)
        return forge_fail(FORGE_INVALID_ARGS, "forge_st_tensor_to_f32: %s holds %lld bytes, not %lld values",
                          v->name ? v->name : "?", (long long)v->nbytes, (long long)n);
    const uint8_t* p = (const uint8_t*)v->data;
    switch (v->dtype) {
        case FORGE_ST_F32: memcpy(out, p, (size_t)n * 4); break;
        case FORGE_ST_BF16:
            for (int64_t i = 0; i < n; ++i) {
                const uint32_t u = (uint32_t)load_le<uint16_t>(p + 2 * i) << 16;
                memcpy(out + i, &u, 4);
            }
            break;
        case FORGE_ST_F16:
            for (int64_t i = 0; i < n; ++i) out[i] = f16_to_f32(load_le<uint16_t>(p + 2 * i));
            break;
        case FORGE_ST_F64:
            for (int64_t i = 0; i < n; ++i) out[i] = (float)load_le<double>(p + 8 * i);
            break;
        default:
            return forge_fail(FORGE_INVALID_ARGS, "forge_st_tensor_to_f32: %s is not a floating-point tensor",
                              v->name ? v->name : "?");
    }
    return 0;
}

// ---- Llama-layout loader ---------------------------------------------------

namespace {
bool is_float_dtype(int dt) {
    return dt == FORGE_ST_BF16 || dt == FORGE_ST_F16 || dt == FORGE_ST_F32 || dt == FORGE_ST_F64;
}

struct Shards {
    std::vector<ForgeSafetensors*> files;
    std::unordered_map<std::string, ForgeStTensor> byname;
    ~Shards() {
        for (ForgeSafetensors* f : files) forge_st_close(f);
    }
    int open(const char* who, int n_files, const char* const* paths) {
        if (n_files <= 0 || !paths) return forge_fail(FORGE_INVALID_ARGS, "%s: no files", who);
        for (int i = 0; i < n_files; ++i) {
            ForgeSafetensors* st = nullptr;
            if (forge_st_open(paths[i], &st)) return FORGE_INVALID_ARGS;
            files.push_back(st);
            for (int t = 0; t < forge_st_count(st); ++t) {
                ForgeStTensor v;
                forge_st_tensor_at(st, t, &v);
                if (!byname.emplace(v.name, v).second)
                    return forge_fail(FORGE_INVALID_ARGS, "%s: %s appears in two files", who, v.name);
            }
        }
        return 0;
    }
};

// One tensor the loader reads: its name and its 1-D (cols 0) or 2-D shape.
struct Want {
    std::string name;
    int64_t rows, cols;
};

// Every tensor of the Llama layout for the description, in load order:
// per layer the seven projections then the two norms, then the embedding,
// the final norm and (untied) the head.
std::vector<Want> llama_tensors(const ForgeModelDesc& d) {
    const int64_t D = d.d_model, Q = (int64_t)d.n_head * d.head_dim, KV = (int64_t)d.n_kv_head * d.head_dim;
    const int64_t F = d.ffn, V = d.vocab;
    static const char* kProj[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                   "mlp.gate_proj",    "mlp.up_proj",      "mlp.down_proj"};
    const int64_t rows[7] = {Q, KV, KV, D, F, F, D}, cols[7] = {D, D, D, Q, D, D, F};
    std::vector<Want> w;
    for (int l = 0; l < d.n_layer; ++l) {
        const std::string pre = "model.layers." + std::to_string(l) + ".";
        for (int i = 0; i < 7; ++i) w.push_back({pre + kProj[i] + ".weight", rows[i], cols[i]});
        w.push_back({pre + "input_layernorm.weight", D, 0});
        w.push_back({pre + "post_attention_layernorm.weight", D, 0});
    }
    w.push_back({"model.embed_tokens.weight", V, D});
    w.push_back({"model.norm.weight", D, 0});
    if (!d.tied_head) w.push_back({"lm_head.weight", V, D});
    return w;
}

int check_one(const Shards& s, const char* who, const Want& w) {
    auto it = s.byname.find(w.name);
    if (it == s.byname.end()) return forge_fail(FORGE_INVALID_ARGS, "%s: %s missing", who, w.name.c_str());
    const ForgeStTensor& v = it->second;
    const bool ok = w.cols ? (v.ndim == 2 && v.shape[0] == w.rows && v.shape[1] == w.cols)
                           : (v.ndim == 1 && v.shape[0] == w.rows);
    if (!ok)
        return forge_fail(FORGE_INVALID_ARGS, "%s: %s has shape [%lld%s%lld], expected [%lld%s%lld]", who,
                          w.name.c_str(), v.ndim > 0 ? (long long)v.shape[0] : 0LL, v.ndim > 1 ? ", " : "",
                          v.ndim > 1 ? (long long)v.shape[1] : 0LL, (long long)w.rows, w.cols ? ", " : "",
                          (long long)w.cols);
    if (!is_float_dtype(v.dtype))
        return forge_fail(FORGE_INVALID_ARGS, "%s: %s is not a floating-point tensor", who, w.name.c_str());
    return 0;
}

// The (checked) tensor converted into bf16 or fp32.
int fetch(const Shards& s, const Want& w, std::vector<uint16_t>* bf, std::vector<float>* f32) {
    const ForgeStTensor& v = s.byname.at(w.name);
    const int64_t n = w.rows * (w.cols ? w.cols : 1);
    if (bf) {
        bf->resize((size_t)n);
        return forge_st_tensor_to_bf16(&v, bf->data(), n);
    }
    f32->resize((size_t)n);
    return forge_st_tensor_to_f32(&v, f32->data(), n);
}
}  // namespace

FORGE_API int forge_safetensors_check_llama(const ForgeModelDesc* d, int n_files, const char* const* paths) {
    const char* who = "forge_safetensors_check_llama";
    if (!d || d->n_layer <= 0 || d->d_model <= 0 || d->n_head <= 0 || d->n_kv_head <= 0 || d->head_dim <= 0 ||
        d->ffn <= 0 || d->vocab <= 0)
        return forge_fail(FORGE_INVALID_ARGS, "%s: bad model description", who);
    Shards s;
    if (s.open(who, n_files, paths)) return FORGE_INVALID_ARGS;
    for (const Want& w : llama_tensors(*d))
        if (check_one(s, who, w)) return FORGE_INVALID_ARGS;
    return 0;
}

FORGE_API int forge_b200_load_safetensors(ForgeB200* h, int n_files, const char* const* paths) {
    const char* who = "forge_b200_load_safetensors";
    const ForgeModelDesc* d = forge_b200_desc_of(h);
    if (!d) return forge_fail(FORGE_INVALID_ARGS, "%s: null handle", who);
    Shards s;
    if (s.open(who, n_files, paths)) return FORGE_INVALID_ARGS;
    const std::vector<Want> want = llama_tensors(*d);
    for (const Want& w : want)  // everything is checked before anything is uploaded
        if (check_one(s, who, w)) return FORGE_INVALID_ARGS;
    std::vector<uint16_t> wb[7];
    std::vector<float> g1, g2;
    size_t k = 0;
    for (int l = 0; l < d->n_layer; ++l) {
        for (int i = 0; i < 7; ++i)
            if (fetch(s, want[k++], &wb[i], nullptr)) return FORGE_INVALID_ARGS;
        if (fetch(s, want[k++], nullptr, &g1) || fetch(s, want[k++], nullptr, &g2)) return FORGE_INVALID_ARGS;
        ForgeLayerWeights lw{wb[0].data(), wb[1].data(), wb[2].data(), wb[3].data(), wb[4].data(),
                             wb[5].data(), wb[6].data(), g1.data(),  g2.data()};
        if (forge_b200_load_layer(h, l, &lw)) return FORGE_INVALID_ARGS;
    }
    std::vector<uint16_t> emb, head;
    std::vector<float> gF;
    if (fetch(s, want[k++], &emb, nullptr) || fetch(s, want[k++], nullptr, &gF)) return FORGE_INVALID_ARGS;
    if (!d->tied_head && fetch(s, want[k++], &head, nullptr)) return FORGE_INVALID_ARGS;
    return forge_b200_load_embedding(h, emb.data(), gF.data(), d->tied_head ? nullptr : head.data());
}
