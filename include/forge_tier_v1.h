/* forge_tier_v1.h — forge's v1 dispatch ABI, kept byte-compatible.
 *
 * Same constants, struct layouts and entry points as the reference header
 * self/forge/forge_tier_v1.h:24-130, restated here so that callers built
 * against the reference link unchanged against libforge_b200.so. The v1
 * contract (caller-owned farrs, no hidden allocation, FORGE_* return codes)
 * is frozen; new kernel families live in forge_b200.h (_v2).
 */
#ifndef FORGE_TIER_V1_H
#define FORGE_TIER_V1_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define FORGE_API_VERSION_V1_MAJOR  1
#define FORGE_API_VERSION_V1_MINOR  0
#define FORGE_API_VERSION_V1_ENCODED \
    ((uint32_t)((FORGE_API_VERSION_V1_MAJOR << 16) | FORGE_API_VERSION_V1_MINOR))

/* kernel families (reference :33-43) */
#define FORGE_KERNEL_MATMUL            1
#define FORGE_KERNEL_FFN_FUSED         2
#define FORGE_KERNEL_FWD_BWD_LINEAR    3
#define FORGE_KERNEL_ATTN_DT_FWD       4
#define FORGE_KERNEL_ATTN_DT_BWD       5
#define FORGE_KERNEL_RMSNORM_MH        6
#define FORGE_KERNEL_SILU_GATE         7
#define FORGE_KERNEL_ROPE_MH           8

/* regime hints (reference :45-50) */
#define FORGE_REGIME_AUTO              0
#define FORGE_REGIME_SMALL             1
#define FORGE_REGIME_MEDIUM            2
#define FORGE_REGIME_LARGE             3

/* precision policy (reference :52-56) */
#define FORGE_PREC_FP64                  0
#define FORGE_PREC_LAYERCAST_BF16_FP32   1
#define FORGE_PREC_PURE_BF16             2

/* determinism mode (reference :58-60) */
#define FORGE_DET_DEFAULT              0
#define FORGE_DET_PEDANTIC             1

/* return codes (reference :62-69) */
#define FORGE_OK                       0
#define FORGE_FALLBACK_USED            1
#define FORGE_KERNEL_UNSUPPORTED      (-1)
#define FORGE_REGIME_UNSUPPORTED      (-2)
#define FORGE_PRECISION_UNSUPPORTED   (-3)
#define FORGE_INVALID_ARGS            (-4)
#define FORGE_ABI_MISMATCH            (-5)

/* shape descriptor (reference :71-79) */
typedef struct ForgeShapeInfo {
    int64_t M;
    int64_t N;
    int64_t K;
    int64_t batch;
} ForgeShapeInfo;

/* farr id bundle (reference :80-101): BF16 precisions carry descriptor
 * pointers cast through intptr_t in each slot. */
typedef struct ForgeArgs {
    int64_t farr_ids[8];
    int     count;
} ForgeArgs;

/* reference :105-108 */
uint32_t forge_api_version_v1(void);

/* reference :110-121 */
int forge_tier_dispatch_v1(int kernel_family, const ForgeShapeInfo* shape, int regime_hint,
                           int precision_policy, int det_mode, const ForgeArgs* in,
                           const ForgeArgs* out);

/* reference :123-130 */
int forge_register_specialized_v1(int kernel_family, const ForgeShapeInfo* shape,
                                  int precision_policy, int regime_hint, void* fn_ptr);

#ifdef __cplusplus
}
#endif
#endif
