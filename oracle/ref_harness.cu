// ref_harness.cu — exposes the reference's own f64 single-layer decode
// reference `cpu_ref` (tool/decode_eager_baseline.cu:160-198) and its input
// LCG (tool/decode_eager_baseline.cu:53-54) through a C ABI. The reference
// file is #included from where it lies (path given by FORGE_REF_SRC); its
// main() is renamed so it never runs. Test infrastructure only.
#define main forge_ref_unused_main
#include FORGE_REF_SRC
#undef main

extern "C" {
int ref_dims(int* d, int* nh, int* hd, int* ff) { *d = D; *nh = NH; *hd = HD; *ff = FF; return 0; }

// Generates the file's inputs in the order its main() draws them
// (tool/decode_eager_baseline.cu:209-219) for cache length L.
void ref_make_inputs(int L, float* x, float* g1, float* g2, float* Wq, float* Wk,
                     float* Wv, float* Wo, float* Wg, float* Wu, float* Wd,
                     float* Kc, float* Vc) {
  lcg = 0x12345678u;
  float wq = 0.036f;
  for (int i = 0; i < D; i++) { x[i] = lcg_f32(); g1[i] = 1.f + 0.1f * lcg_f32(); g2[i] = 1.f + 0.1f * lcg_f32(); }
  for (int i = 0; i < D * D; i++) { Wq[i] = lcg_f32() * wq; Wk[i] = lcg_f32() * wq; Wv[i] = lcg_f32() * wq; Wo[i] = lcg_f32() * wq; }
  for (int i = 0; i < FF * D; i++) { Wg[i] = lcg_f32() * wq; Wu[i] = lcg_f32() * wq; }
  for (int i = 0; i < D * FF; i++) Wd[i] = lcg_f32() * 0.018f;
  for (int i = 0; i < L * D; i++) { Kc[i] = lcg_f32() * wq * 0.5f; Vc[i] = lcg_f32(); }
}

void ref_cpu_ref(const float* x, const float* g1, const float* g2, const float* Wq,
                 const float* Wk, const float* Wv, const float* Wo, const float* Wg,
                 const float* Wu, const float* Wd, const float* Kc, const float* Vc,
                 int L, double* out) {
  cpu_ref(x, g1, g2, Wq, Wk, Wv, Wo, Wg, Wu, Wd, Kc, Vc, L, out);
}
}
