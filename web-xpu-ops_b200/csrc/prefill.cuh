// prefill.cuh — the resident prefill (prefill.cu) as the engine drives it.
#pragma once

#include "common.cuh"

namespace xpu {

struct PrefillLayer {
  const float* attn_norm;
  const float* ffn_norm;
  const uint32_t* wqkv;  // [q; k; v] rows, ldw_h words each
  const float* sqkv;
  const uint32_t* wo;    // ldw_qd words per row
  const float* so;
  const uint32_t* wg;    // ldw_h
  const float* sg;
  const uint32_t* wu;    // ldw_h
  const float* su;
  const uint32_t* wd;    // ldw_f
  const float* sd;
  int64_t ldw_h, ldw_qd, ldw_f;
  float* kcache;
  float* vcache;
};

struct PrefillArgs {
  const PrefillLayer* layer;  // host array [layers]
  int layers, hidden, H, kvH, hd, ffn, vocab, S;
  double eps;
  float attn_scale;
  const int8_t* embed_codes;
  const float* embed_scale;
  const double* inv_freq;
  // activations, [chunk rows] each: hidden, q, attention output, FFN
  float *hid, *hid2, *xn, *qkv, *q, *attn, *gate, *up;
};

// Argument limits of the attention kernel; XPU_OK or XPU_EINVAL.
int prefill_check(int H, int kvH, int hd);
// Tokens d_tokens[0, T) (device) at positions [p0, p0 + T) through every
// layer; leaves the last layer's output in a.hid and fills the caches.
int prefill_chunk(const PrefillArgs& a, const int32_t* d_tokens, int T, int p0, cudaStream_t st);

}  // namespace xpu
