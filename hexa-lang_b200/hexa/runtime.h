/* runtime.h — the part of the hexa runtime interface that C emitted by the
 * hexa transpiler (hexat) from forge_greedy.hexa calls: tagged values,
 * integer / float / string arithmetic and comparison, printing, exit, raw memory
 * (alloc_raw / ptr_read / ptr_write and their 32-bit forms) and the @link
 * symbol loader. The names and signatures are those the emitted code calls
 * (hexa-lang's self/runtime.h declares the full runtime); the definitions
 * in hexa_shim.c are this library's own, just enough to run a flame driver
 * of the forge_b200 engine without hexa-lang's runtime.c. */
#ifndef FORGE_HEXA_RUNTIME_H
#define FORGE_HEXA_RUNTIME_H
#include <stdint.h>
#include <stdio.h>

enum { HX_T_VOID = 0, HX_T_INT = 1, HX_T_FLOAT = 2, HX_T_BOOL = 3, HX_T_STR = 4 };

typedef struct HexaVal {
    int32_t tag;
    union {
        int64_t i;
        double f;
        const char* s;
    } u;
} HexaVal;

#define HX_IS_INT(v) ((v).tag == HX_T_INT || (v).tag == HX_T_BOOL)
#define HX_IS_FLOAT(v) ((v).tag == HX_T_FLOAT)
#define HX_INT(v) ((v).u.i)
#define HX_INT_U(v) ((v).u.i)
#define HX_FLOAT(v) ((v).tag == HX_T_FLOAT ? (v).u.f : (double)(v).u.i)
#define HX_BOOL(v) ((v).u.i != 0)

HexaVal hexa_int(int64_t n);
HexaVal hexa_float(double x);
HexaVal hexa_bool(int b);
HexaVal hexa_str(const char* s);
HexaVal hexa_void(void);

HexaVal hexa_add(HexaVal a, HexaVal b);
HexaVal hexa_sub(HexaVal a, HexaVal b);
HexaVal hexa_mul(HexaVal a, HexaVal b);
HexaVal hexa_cmp_lt(HexaVal a, HexaVal b);
HexaVal hexa_cmp_gt(HexaVal a, HexaVal b);
HexaVal hexa_eq(HexaVal a, HexaVal b);
int hexa_truthy(HexaVal v);
HexaVal hexa_to_string(HexaVal v);
void hexa_println(HexaVal v);

HexaVal hexa_ptr_alloc(HexaVal size);
HexaVal hexa_ptr_free(HexaVal ptr, HexaVal size);
HexaVal hexa_ptr_read(HexaVal ptr, HexaVal offset);
HexaVal hexa_ptr_write(HexaVal ptr, HexaVal offset, HexaVal val);
HexaVal hexa_ptr_read_i32(HexaVal ptr, HexaVal offset);
HexaVal hexa_ptr_write_i32(HexaVal ptr, HexaVal offset, HexaVal val);

void __hexa_fn_arena_enter(void);
HexaVal __hexa_fn_arena_return(HexaVal ret);
void hexa_set_args(int argc, char** argv);
HexaVal hexa_exit(HexaVal code);

void* hexa_ffi_dlopen(const char* lib_name);
void* hexa_ffi_dlsym(void* handle, const char* symbol);
#endif
