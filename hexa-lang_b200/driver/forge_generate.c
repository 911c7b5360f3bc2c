/* forge_generate.c — command-line generation through the C ABI of
 * libforge_b200.so: the C greedy-loop caller of the decode path.
 *
 * It follows the shape of the reference's generation loop
 * (self/ml/gpu_generate.hexa:1-20: initialise, load or randomly initialise
 * the weights, feed the prompt through the KV cache, decode token by token,
 * report tok/s) and its sampler settings (self/ml/gpu_sampler.hexa:23-47:
 * temperature <= 0 is greedy). Only public entries of include/ are used.
 *
 *   forge_generate --layers L --dim D --heads H --kv-heads HKV --head-dim HD
 *                  --ffn F --vocab V [--int4] [--tied] [--ctx N] [--device G]
 *                  [--weights a.safetensors[,b.safetensors...] | --synthetic SEED]
 *                  [--temperature T] [--top-k K] [--top-p P] [--seed S]
 *                  --gen N  TOKEN [TOKEN ...]
 *   forge_generate --check <model options> --weights a.safetensors[,...]
 *
 * --check only validates the checkpoint against the model options (every
 * tensor present, shaped and typed as the loader needs it); no GPU is used.
 *
 * Prints the N generated token ids on one line (stdout) and the decode rate
 * on stderr. Exit status 0 on success, 1 on a library error (its message on
 * stderr), 2 on bad usage.
 */
#define _POSIX_C_SOURCE 200809L
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "forge_b200.h"
#include "forge_safetensors.h"

static void usage(FILE* f) {
    fprintf(f,
            "usage: forge_generate --layers L --dim D --heads H --kv-heads HKV --head-dim HD --ffn F --vocab V\n"
            "                      [--int4] [--tied] [--ctx N] [--device G]\n"
            "                      [--weights a.safetensors[,b...] | --synthetic SEED]\n"
            "                      [--temperature T] [--top-k K] [--top-p P] [--seed S] --gen N TOKEN...\n"
            "       forge_generate --check <model options> --weights a.safetensors[,b...]\n");
}

static int fail(ForgeB200* h, const char* what) {
    fprintf(stderr, "forge_generate: %s: %s\n", what, forge_b200_last_error());
    if (h) forge_b200_destroy(h);
    return 1;
}

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

int main(int argc, char** argv) {
    ForgeModelDesc d;
    memset(&d, 0, sizeof d);
    d.rms_eps = 1e-5f;
    d.rope_theta = 10000.0f;
    d.max_batch = 1;
    d.max_ctx = 0;
    d.tp_size = 1;
    int device = 0, n_gen = 0, top_k = 0;
    double temperature = 0.0, top_p = 1.0;
    long long seed = 42, synth = -1;
    char* weights = NULL;
    int check_only = 0;
    int32_t* prompt = NULL;
    int n_prompt = 0;
    for (int i = 1; i < argc; ++i) {
        const char* a = argv[i];
        const int more = i + 1 < argc;
#define INTARG(flag, dst)                           \
    if (!strcmp(a, flag)) {                         \
        if (!more) { usage(stderr); return 2; }     \
        dst = atoi(argv[++i]);                      \
        continue;                                   \
    }
        if (!strcmp(a, "--help") || !strcmp(a, "-h")) {
            usage(stdout);
            return 0;
        }
        INTARG("--layers", d.n_layer)
        INTARG("--dim", d.d_model)
        INTARG("--heads", d.n_head)
        INTARG("--kv-heads", d.n_kv_head)
        INTARG("--head-dim", d.head_dim)
        INTARG("--ffn", d.ffn)
        INTARG("--vocab", d.vocab)
        INTARG("--ctx", d.max_ctx)
        INTARG("--device", device)
        INTARG("--gen", n_gen)
        INTARG("--top-k", top_k)
#undef INTARG
        if (!strcmp(a, "--int4")) { d.weight_kind = FORGE_WEIGHT_Q4_G128; continue; }
        if (!strcmp(a, "--tied")) { d.tied_head = 1; continue; }
        if (!strcmp(a, "--check")) { check_only = 1; continue; }
        if (more && !strcmp(a, "--temperature")) { temperature = atof(argv[++i]); continue; }
        if (more && !strcmp(a, "--top-p")) { top_p = atof(argv[++i]); continue; }
        if (more && !strcmp(a, "--seed")) { seed = atoll(argv[++i]); continue; }
        if (more && !strcmp(a, "--synthetic")) { synth = atoll(argv[++i]); continue; }
        if (more && !strcmp(a, "--weights")) { weights = argv[++i]; continue; }
        if (a[0] == '-' && (a[1] < '0' || a[1] > '9')) {
            fprintf(stderr, "forge_generate: unknown option %s\n", a);
            usage(stderr);
            return 2;
        }
        int32_t* p = (int32_t*)realloc(prompt, sizeof(int32_t) * (size_t)(n_prompt + 1));
        if (!p) return 2;
        prompt = p;
        prompt[n_prompt++] = (int32_t)atoi(a);
    }
    if (check_only) {
        if (!weights || d.n_layer <= 0 || d.d_model <= 0 || d.n_head <= 0 || d.n_kv_head <= 0 || d.head_dim <= 0 ||
            d.ffn <= 0 || d.vocab <= 0) {
            usage(stderr);
            free(prompt);
            return 2;
        }
        const char* paths[64];
        int n = 0;
        for (char* s = strtok(weights, ","); s && n < 64; s = strtok(NULL, ",")) paths[n++] = s;
        free(prompt);
        if (forge_safetensors_check_llama(&d, n, paths)) return fail(NULL, "check");
        printf("ok: %d file(s) hold every tensor of the model\n", n);
        return 0;
    }
    if (d.n_layer <= 0 || d.d_model <= 0 || d.n_head <= 0 || d.n_kv_head <= 0 || d.head_dim <= 0 || d.ffn <= 0 ||
        d.vocab <= 0 || n_gen <= 0 || n_prompt == 0 || (!weights && synth < 0)) {
        usage(stderr);
        free(prompt);
        return 2;
    }
    if (d.max_ctx <= 0) d.max_ctx = n_prompt + n_gen;

    ForgeB200* h = NULL;
    if (forge_b200_create(&d, device, &h)) { free(prompt); return fail(NULL, "create"); }
    if (weights) {
        const char* paths[64];
        int n = 0;
        for (char* s = strtok(weights, ","); s && n < 64; s = strtok(NULL, ",")) paths[n++] = s;
        if (forge_b200_load_safetensors(h, n, paths)) { free(prompt); return fail(h, "load_safetensors"); }
    } else if (forge_b200_init_synthetic(h, (uint64_t)synth, 0.02f)) {
        free(prompt);
        return fail(h, "init_synthetic");
    }

    int32_t* out = (int32_t*)malloc(sizeof(int32_t) * (size_t)n_gen);
    const double t0 = now_s();
    int rc = 0;
    if (temperature <= 0.0) {
        rc = forge_b200_generate(h, 1, prompt, n_prompt, n_gen, out);
    } else {
        /* prompt through the KV cache, then one sampled token per step */
        int64_t state = (int64_t)seed;
        int32_t cur = prompt[0], next = 0;
        rc = forge_b200_reset(h);
        for (int p = 0; p + 1 < n_prompt && !rc; ++p) {
            rc = forge_b200_decode_step(h, 1, &prompt[p], &next, NULL);
        }
        cur = prompt[n_prompt - 1];
        for (int i = 0; i < n_gen && !rc; ++i) {
            rc = forge_b200_decode_step_sampled(h, 1, &cur, &next, temperature, top_k, top_p, &state);
            out[i] = next;
            cur = next;
        }
    }
    const double dt = now_s() - t0;
    free(prompt);
    if (rc) {
        free(out);
        return fail(h, "decode");
    }
    for (int i = 0; i < n_gen; ++i) printf(i ? " %d" : "%d", out[i]);
    printf("\n");
    fprintf(stderr, "forge_generate: %d tokens in %.3f s (%.1f tok/s, prompt included)\n", n_gen, dt, n_gen / dt);
    free(out);
    forge_b200_destroy(h);
    return 0;
}
