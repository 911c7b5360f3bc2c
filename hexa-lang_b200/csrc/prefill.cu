// prefill.cu — causal flash-attention prefill (v2 FLASH_PREFILL family).
#include "forge_internal.h"
#include "../../include/forge_b200.h"
#include "../../include/forge_farr.h"

int forge_prefill_dispatch(const ForgeShapeInfo* s, const ForgeArgs* in, const ForgeArgs* out) {
    (void)s; (void)in; (void)out;
    forge_fail(FORGE_KERNEL_UNSUPPORTED, "FLASH_PREFILL: not built");
    return FORGE_KERNEL_UNSUPPORTED;
}
