// Host entries of the attention kernels: argument checks, then the tcgen05 kernel of
// attention_tc.cu for every case -- the causal prefill over all rows, the static-FP8-output
// variant, selected query rows (the pick-row tail), and the vision tower's non-causal
// attention over one image -- so that every attention output of the library comes from
// one arithmetic.
//
// Semantics of the reference kernel (_legacy/limit_kernels.py:8-33): scores in fp32,
// scaled by 1/sqrt(128); online softmax over 64-key blocks (running max, rescaled
// accumulator); the probabilities are cast to bf16 before the P.V product; output
// bf16(acc / den).  Keys n > position are masked (position = query index, or the
// explicit `positions` of the tail's selected rows).
#include "common.cuh"

int ffb_attention_tc(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int64_t* sel, int q_gather,
                     int S, const int* key_lo, void* out, int T, int HQ, int HK, float scale, float out_inv,
                     int causal, int out_cols, void* rq_sync, float* qscale, cudaStream_t stream);

extern "C" int ffb_attention_segmented(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                       const int64_t* positions, int q_gather, const int* key_lo, uint16_t* out, int S,
                                       int T, int HQ, int HK, float scale, void* stream) {
  FFB_REQUIRE(q && k && v && out, "ffb_attention: NULL pointer");
  FFB_REQUIRE(S > 0 && T > 0 && HQ > 0 && HK > 0 && HQ % HK == 0, "ffb_attention: bad shape S=%d T=%d HQ=%d HK=%d", S,
              T, HQ, HK);
  FFB_REQUIRE(positions || S == T, "ffb_attention: causal prefill needs S == T (or explicit positions)");
  FFB_REQUIRE(!q_gather || positions, "ffb_attention: q_gather needs positions");
  FFB_REQUIRE(ffb::aligned(q, 16) && ffb::aligned(k, 16) && ffb::aligned(v, 16) && ffb::aligned(out, 16),
              "ffb_attention: q, k, v and out must be 16-byte aligned");
  FFB_REQUIRE(!key_lo || ffb::aligned(key_lo, 4), "ffb_attention: key_lo alignment");
  FFB_REQUIRE(!positions || ffb::aligned(positions, 8), "ffb_attention: positions alignment");
  return ffb_attention_tc(q, k, v, positions, q_gather, S, key_lo, out, T, HQ, HK, scale, 0.f, 1, 0, nullptr,
                          nullptr, (cudaStream_t)stream);
}

extern "C" int ffb_attention_fp8(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int* key_lo,
                                 float out_inv, uint8_t* out8, int T, int HQ, int HK, float scale, void* stream) {
  FFB_REQUIRE(q && k && v && out8, "ffb_attention_fp8: NULL pointer");
  FFB_REQUIRE(T > 0 && HQ > 0 && HK > 0 && HQ % HK == 0, "ffb_attention_fp8: bad shape T=%d HQ=%d HK=%d", T, HQ, HK);
  FFB_REQUIRE(out_inv > 0.f, "ffb_attention_fp8: out_inv must be positive");
  FFB_REQUIRE(ffb::aligned(q, 16) && ffb::aligned(k, 16) && ffb::aligned(v, 16) && ffb::aligned(out8, 16),
              "ffb_attention_fp8: alignment");
  FFB_REQUIRE(!key_lo || ffb::aligned(key_lo, 4), "ffb_attention_fp8: key_lo alignment");
  return ffb_attention_tc(q, k, v, nullptr, 0, T, key_lo, out8, T, HQ, HK, scale, out_inv, 1, 0, nullptr, nullptr,
                          (cudaStream_t)stream);
}

extern "C" int ffb_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int64_t* positions,
                             int q_gather, uint16_t* out, int S, int T, int HQ, int HK, float scale, void* stream) {
  return ffb_attention_segmented(q, k, v, positions, q_gather, nullptr, out, S, T, HQ, HK, scale, stream);
}

extern "C" int ffb_attention_full(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int T,
                                  int H, int d, float scale, void* stream) {
  FFB_REQUIRE(q && k && v && out, "ffb_attention_full: NULL pointer");
  FFB_REQUIRE(T > 0 && H > 0, "ffb_attention_full: bad shape T=%d H=%d", T, H);
  FFB_REQUIRE(d > 0 && d <= 128 && d % 8 == 0, "ffb_attention_full: head dim %d (8..128, a multiple of 8)", d);
  FFB_REQUIRE(ffb::aligned(q, 16) && ffb::aligned(k, 16) && ffb::aligned(v, 16) && ffb::aligned(out, 16),
              "ffb_attention_full: q, k, v and out must be 16-byte aligned");
  return ffb_attention_tc(q, k, v, nullptr, 0, T, nullptr, out, T, H, H, scale, 0.f, 0, d, nullptr, nullptr,
                          (cudaStream_t)stream);
}

extern "C" int ffb_attention_rowwise_sync_bytes(int T, int HQ) {
  return T > 0 && HQ > 0 ? 4 * T * HQ + 4 * ((T + 127) / 128) : 0;
}

extern "C" int ffb_attention_rowwise(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint8_t* out8,
                                     float* qscale, void* sync, int T, int HQ, int HK, float scale, void* stream) {
  FFB_REQUIRE(q && k && v && out8 && qscale && sync, "ffb_attention_rowwise: NULL pointer");
  FFB_REQUIRE(T > 0 && HQ > 0 && HK > 0 && HQ % HK == 0 && HQ % 4 == 0,
              "ffb_attention_rowwise: bad shape T=%d HQ=%d HK=%d (HQ a multiple of 4)", T, HQ, HK);
  FFB_REQUIRE(ffb::aligned(q, 16) && ffb::aligned(k, 16) && ffb::aligned(v, 16) && ffb::aligned(out8, 16) &&
                  ffb::aligned(sync, 16) && ffb::aligned(qscale, 4),
              "ffb_attention_rowwise: alignment");
  const long long ctas = (long long)((T + 127) / 128) * HQ;
  if (ctas > ffb::sm_count())
    return ffb::fail(FFB_EUNSUPPORTED,
                     "ffb_attention_rowwise: %lld CTAs exceed the %d SMs (the row maxima need every CTA resident)",
                     ctas, ffb::sm_count());
  return ffb_attention_tc(q, k, v, nullptr, 0, T, nullptr, out8, T, HQ, HK, scale, 0.f, 1, 0, sync, qscale,
                          (cudaStream_t)stream);
}
