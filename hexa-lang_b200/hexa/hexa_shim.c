/* hexa_shim.c — definitions of the hexa runtime calls declared in runtime.h,
 * enough to run a transpiled flame driver of forge_b200 (see runtime.h).
 * Semantics follow hexa's: ints are 64-bit; `+` adds numbers and
 * concatenates when either side is a string; alloc_raw returns a raw
 * address as an int; ptr_write stores 8 bytes (an int as int64, a float as
 * its IEEE-754 double bits, as hexa's packed-argument FFI blocks expect);
 * ptr_read loads an int64; the _i32 forms store / load 4-byte ints.
 * @link("name") resolves lib<name>.so through the dynamic loader's search
 * path (LD_LIBRARY_PATH), and a missing library or symbol ends the program
 * with one line on stderr, as the hexa runtime's loader does. Strings live
 * until exit (the program is short-lived; no garbage collector here). */
#include "runtime.h"

#include <dlfcn.h>
#include <inttypes.h>
#include <stdlib.h>
#include <string.h>

HexaVal hexa_int(int64_t n) {
    HexaVal v;
    v.tag = HX_T_INT;
    v.u.i = n;
    return v;
}
HexaVal hexa_float(double x) {
    HexaVal v;
    v.tag = HX_T_FLOAT;
    v.u.f = x;
    return v;
}
HexaVal hexa_bool(int b) {
    HexaVal v;
    v.tag = HX_T_BOOL;
    v.u.i = b != 0;
    return v;
}
HexaVal hexa_str(const char* s) {
    HexaVal v;
    v.tag = HX_T_STR;
    v.u.s = s;
    return v;
}
HexaVal hexa_void(void) {
    HexaVal v;
    v.tag = HX_T_VOID;
    v.u.i = 0;
    return v;
}

static const char* fmt_val(HexaVal v) {
    char buf[64];
    switch (v.tag) {
    case HX_T_STR: return v.u.s;
    case HX_T_FLOAT: snprintf(buf, sizeof buf, "%.17g", v.u.f); break;
    case HX_T_BOOL: return v.u.i ? "true" : "false";
    case HX_T_VOID: return "void";
    default: snprintf(buf, sizeof buf, "%" PRId64, v.u.i); break;
    }
    char* s = strdup(buf);
    if (!s) {
        fprintf(stderr, "hexa: out of memory\n");
        exit(2);
    }
    return s;
}

HexaVal hexa_add(HexaVal a, HexaVal b) {
    if (a.tag == HX_T_STR || b.tag == HX_T_STR) {
        const char *x = fmt_val(a), *y = fmt_val(b);
        size_t n = strlen(x) + strlen(y) + 1;
        char* s = (char*)malloc(n);
        if (!s) {
            fprintf(stderr, "hexa: out of memory\n");
            exit(2);
        }
        snprintf(s, n, "%s%s", x, y);
        return hexa_str(s);
    }
    if (HX_IS_FLOAT(a) || HX_IS_FLOAT(b)) return hexa_float(HX_FLOAT(a) + HX_FLOAT(b));
    return hexa_int(a.u.i + b.u.i);
}
HexaVal hexa_sub(HexaVal a, HexaVal b) {
    if (HX_IS_FLOAT(a) || HX_IS_FLOAT(b)) return hexa_float(HX_FLOAT(a) - HX_FLOAT(b));
    return hexa_int(a.u.i - b.u.i);
}
HexaVal hexa_mul(HexaVal a, HexaVal b) {
    if (HX_IS_FLOAT(a) || HX_IS_FLOAT(b)) return hexa_float(HX_FLOAT(a) * HX_FLOAT(b));
    return hexa_int(a.u.i * b.u.i);
}
HexaVal hexa_cmp_lt(HexaVal a, HexaVal b) {
    if (HX_IS_FLOAT(a) || HX_IS_FLOAT(b)) return hexa_bool(HX_FLOAT(a) < HX_FLOAT(b));
    return hexa_bool(a.u.i < b.u.i);
}
HexaVal hexa_cmp_gt(HexaVal a, HexaVal b) { return hexa_cmp_lt(b, a); }
HexaVal hexa_eq(HexaVal a, HexaVal b) {
    if (a.tag == HX_T_STR && b.tag == HX_T_STR) return hexa_bool(strcmp(a.u.s, b.u.s) == 0);
    if (a.tag == HX_T_STR || b.tag == HX_T_STR) return hexa_bool(0);
    if (HX_IS_FLOAT(a) || HX_IS_FLOAT(b)) return hexa_bool(HX_FLOAT(a) == HX_FLOAT(b));
    return hexa_bool(a.u.i == b.u.i);
}
int hexa_truthy(HexaVal v) {
    switch (v.tag) {
    case HX_T_VOID: return 0;
    case HX_T_FLOAT: return v.u.f != 0.0;
    case HX_T_STR: return v.u.s && v.u.s[0];
    default: return v.u.i != 0;
    }
}
HexaVal hexa_to_string(HexaVal v) { return hexa_str(fmt_val(v)); }
void hexa_println(HexaVal v) { printf("%s\n", fmt_val(v)); }

HexaVal hexa_ptr_alloc(HexaVal size) {
    void* p = calloc(1, (size_t)(size.u.i > 0 ? size.u.i : 1));
    if (!p) {
        fprintf(stderr, "hexa: alloc_raw(%" PRId64 ") failed\n", size.u.i);
        exit(2);
    }
    return hexa_int((int64_t)(uintptr_t)p);
}
HexaVal hexa_ptr_free(HexaVal ptr, HexaVal size) {
    (void)size;
    free((void*)(uintptr_t)ptr.u.i);
    return hexa_void();
}
HexaVal hexa_ptr_read(HexaVal ptr, HexaVal offset) {
    int64_t v;
    memcpy(&v, (const char*)(uintptr_t)ptr.u.i + offset.u.i, 8);
    return hexa_int(v);
}
HexaVal hexa_ptr_write(HexaVal ptr, HexaVal offset, HexaVal val) {
    char* dst = (char*)(uintptr_t)ptr.u.i + offset.u.i;
    if (HX_IS_FLOAT(val)) {
        double f = val.u.f;
        memcpy(dst, &f, 8);
    } else {
        memcpy(dst, &val.u.i, 8);
    }
    return hexa_void();
}
HexaVal hexa_ptr_read_i32(HexaVal ptr, HexaVal offset) {
    int32_t v;
    memcpy(&v, (const char*)(uintptr_t)ptr.u.i + offset.u.i, 4);
    return hexa_int(v);
}
HexaVal hexa_ptr_write_i32(HexaVal ptr, HexaVal offset, HexaVal val) {
    int32_t v = (int32_t)(HX_IS_FLOAT(val) ? (int64_t)val.u.f : val.u.i);
    memcpy((char*)(uintptr_t)ptr.u.i + offset.u.i, &v, 4);
    return hexa_void();
}

void __hexa_fn_arena_enter(void) {}
HexaVal __hexa_fn_arena_return(HexaVal ret) { return ret; }

static int g_argc;
static char** g_argv;
void hexa_set_args(int argc, char** argv) {
    g_argc = argc;
    g_argv = argv;
}

HexaVal hexa_exit(HexaVal code) {
    fflush(stdout);
    fflush(stderr);
    exit((int)code.u.i);
}

void* hexa_ffi_dlopen(const char* lib_name) {
    char path[512];
    snprintf(path, sizeof path, "lib%s.so", lib_name);
    void* h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        fprintf(stderr, "hexa: @link(\"%s\"): %s\n", lib_name, dlerror());
        exit(2);
    }
    return h;
}
void* hexa_ffi_dlsym(void* handle, const char* symbol) {
    void* s = dlsym(handle, symbol);
    if (!s) {
        fprintf(stderr, "hexa: extern fn %s: %s\n", symbol, dlerror());
        exit(2);
    }
    return s;
}
