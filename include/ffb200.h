/*
 * ffb200.h - C ABI of libffb200.so, the B200 (sm_100a) kernels behind FastForward's
 * Qwen3-VL language-decoder prefill + choice-scoring path.
 *
 * Every entry point replaces one fused op of the reference (FastForward 0.2.4.post1,
 * paths relative to src/fastforward_accel/), cited beside it.  Conventions:
 *   - all tensor arguments are caller-owned device pointers; bf16 tensors are passed
 *     as raw 16-bit words (uint16_t), FP8 e4m3 as uint8_t, row-major unless stated;
 *   - `stream` is a cudaStream_t passed as void*; work is enqueued on it and the call
 *     returns without synchronising; no entry point allocates device memory: scratch
 *     space is passed in (`ws`), except for ffb_quantize_weight_fp8_noalloc, which uses
 *     a fixed array inside the library;
 *   - return value 0 on success, a negative FFB_E* code otherwise; the message of the
 *     last failure on the calling thread is available from ffb_last_error();
 *   - reentrant: the only mutable global state is a per-device error word that kernels
 *     set when a bounded device-side wait gives up (read with ffb_device_error()).
 */
#ifndef FFB200_H
#define FFB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FFB_OK 0
#define FFB_EINVAL (-1)        /* bad shape / pointer / alignment / argument        */
#define FFB_EUNSUPPORTED (-2)  /* a configuration the kernels do not implement      */
#define FFB_ECUDA (-3)         /* a CUDA runtime / driver call failed               */
#define FFB_ETIMEOUT (-4)      /* a kernel's bounded wait gave up (device error word) */

/* Activation quantisation modes of the FP8 path. */
#define FFB_QUANT_NONE 0       /* no FP8 output                                           */
#define FFB_QUANT_STATIC 1     /* q = e4m3(clamp(x * inv, +-448)); depth_fp8.py:8-12       */
#define FFB_QUANT_ROWWISE 2    /* s = max|x_row|/448, q = e4m3(x / s); fp8_private.py:11-18 */
#define FFB_QUANT_ROWSCALE 3   /* ffb_quantize_fp8 only: q = e4m3(clamp(x / s)) with s = qscale[row]
                                  given (a row split over tensor-parallel ranks: the whole row's
                                  ROWWISE scale, the MAX over the ranks' slice scales)          */

/* GEMM epilogues. */
#define FFB_EPI_BF16 0         /* out[m,n] = bf16(acc * sa * sw)                           */
#define FFB_EPI_F32_PARTIAL 1  /* ws[split][m][n] = acc * sa * sw (fp32), reduced by the consumer */
#define FFB_EPI_SWIGLU 2       /* gate/up rows interleaved per 128; out[m,c] = bf16(bf16(silu(g)) * u) */

/* Epilogues of the bf16 linear (ffb_bf16_gemm); v = fp32(acc + bias[n]) (bias NULL: 0). */
#define FFB_EPI_BIAS 10            /* out = bf16(v)                                        */
#define FFB_EPI_BIAS_RES 11        /* out = bf16(res + bf16(v)) (res may alias out)        */
#define FFB_EPI_BIAS_GELU_TANH 12  /* out = bf16(gelu_tanh(bf16(v)))                       */
#define FFB_EPI_BIAS_GELU_ERF 13   /* out = bf16(gelu_erf(bf16(v)))                        */

/* Library identification: returns a static string ("ffb200 <version> sm_100a"). */
const char* ffb_version(void);

/* Enables (1) or disables (0) programmatic dependent launch for every kernel launched
 * afterwards (default on): each kernel then overlaps its launch and prologue with the
 * previous kernel on the stream and waits on the device before touching memory.
 * Returns the previous setting.  Process-wide; not a per-call argument. */
int ffb_set_pdl(int enable);

/* Copies the calling thread's last error message into buf (always NUL-terminated). */
int ffb_last_error(char* buf, size_t len);

/* Reads (and with clear != 0, resets) the current device's error word: 0 = no error,
 * else a bit set per kernel family whose bounded wait timed out.  Synchronous. */
int ffb_device_error(uint32_t* word, int clear);

/* Embedding gather + visual-row scatter.
 * Replaces scaled_qwen_runtime.py:145 `embed_tokens(ids).index_copy(1, vi, visual)`.
 * h[t] = table[ids[t]] for t outside [image_start, image_start+nv), visual[t-image_start] inside. */
int ffb_embed_gather(const int64_t* ids, const uint16_t* table, int64_t vocab,
                     const uint16_t* visual, int image_start, int nv,
                     uint16_t* h, int T, int H, void* stream);

/* Plain RMSNorm (+ optional fused FP8 quantisation of the output).
 * Replaces _legacy/sub10_runtime.py:31-41 (`rms_one` / `fast_norm`); the fused quant
 * replaces the quantiser launched by the next linear (_family/depth_fp8.py:15-19 or
 * _legacy/fp8_private.py:11-18).  out may be NULL when only the FP8 copy is wanted.
 * q8 [T,H] e4m3 and qscale [T] fp32 (ROWWISE) are written when quant_mode != NONE. */
int ffb_rmsnorm(const uint16_t* x, const uint16_t* w, float eps, uint16_t* out,
                int quant_mode, float inv_scale, uint8_t* q8, float* qscale,
                int T, int H, void* stream);

/* Residual add (+ deepstack rows) + RMSNorm (+ optional fused FP8 quant).
 * Replaces _legacy/lower_kernels.py:7-32 (`_add_rms` / `add_rms`).
 * b is the bf16 [T,H] branch output, or (b == NULL) the sum over `splits` fp32 partial
 * tiles b32[splits][T][H] that a split-K GEMM left (rounded to bf16 before the add).
 * deep [nv,H] is added to rows [start, start+nv) (NULL for none). */
int ffb_add_rmsnorm(const uint16_t* a, const uint16_t* b, const float* b32, int splits,
                    const uint16_t* deep, int start, int nv,
                    const uint16_t* w, float eps, uint16_t* residual, uint16_t* out,
                    int quant_mode, float inv_scale, uint8_t* q8, float* qscale,
                    int T, int H, void* stream);

/* Per-head QK RMSNorm + interleaved-M-RoPE rotation (rotate-half with bf16 cos/sin).
 * Replaces _legacy/broad_kernels.py:63-74 (`qk_pair`) -> lower_kernels.py:66-98.
 * Input: the packed qkv rows [T, (HQ+2HK)*128] as bf16 (qkv) or as `splits` fp32
 * partials (qkv == NULL, qkv32[splits][T][row_stride]).  Output head-major:
 * yq [HQ,T,128], yk [HK,T,128] and the V copy yv [HK,T,128] (yv may be NULL). */
int ffb_qk_norm_rope(const uint16_t* qkv, const float* qkv32, int splits, int row_stride,
                     const uint16_t* q_norm, const uint16_t* k_norm, float eps,
                     const uint16_t* cos, const uint16_t* sin,
                     uint16_t* yq, uint16_t* yk, uint16_t* yv,
                     int T, int HQ, int HK, void* stream);

/* Causal GQA attention, head_dim 128.
 * Replaces _legacy/limit_kernels.py:36-45 (`attention_direct`, triangular, or SELECTED
 * with `positions`).  k/v [HK,T,128] (head-major, contiguous); positions [S] int64 or
 * NULL (= 0..S-1).  q is [HQ,S,128], or with q_gather != 0 (needs positions) the full
 * [HQ,T,128] projection from which query row s is q[:, positions[s]] (the tail's
 * `q.index_select(2, pick)`, _family/night_runtime.py:100).  out [S, HQ*128] bf16. */
int ffb_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                  const int64_t* positions, int q_gather, uint16_t* out,
                  int S, int T, int HQ, int HK, float scale, void* stream);

/* ffb_attention over a sequence that holds several independent requests one after the
 * other (batched prefill): query row s sees keys [key_lo[s], position of s], where key_lo
 * (int32 [S], device) is the first row of the row's own request (NULL: 0, i.e. ffb_attention).
 * For the causal prefill (positions == NULL) key_lo must be non-decreasing with
 * key_lo[s] <= s.  No counterpart in the reference (it serialises requests,
 * README.md:53); each request's rows get exactly the keys its own ffb_attention call
 * would give them. */
int ffb_attention_segmented(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                            const int64_t* positions, int q_gather, const int* key_lo, uint16_t* out,
                            int S, int T, int HQ, int HK, float scale, void* stream);

/* Causal prefill attention (as ffb_attention_segmented with positions == NULL, S == T)
 * whose output is the STATIC FP8 input of the o projection: out8[t, h*128 + d] =
 * e4m3(clamp(bf16(attention output) * out_inv, +-448)) (u8 [T, HQ*128]), byte-identical to
 * ffb_attention followed by ffb_quantize_fp8 (FFB_QUANT_STATIC, out_inv).  Replaces
 * `attention_direct` (_legacy/limit_kernels.py:36-45) plus the o projection's
 * `_runtime_scale` (_family/depth_fp8.py:8-12) on the static-scale path.  key_lo as in
 * ffb_attention_segmented (NULL: one request); out_inv > 0; out8 16-byte aligned. */
int ffb_attention_fp8(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int* key_lo,
                      float out_inv, uint8_t* out8, int T, int HQ, int HK, float scale, void* stream);

/* Causal prefill attention (as ffb_attention with positions == NULL, S == T) whose output
 * is the ROWWISE FP8 input of the o projection: out8 [T, HQ*128] e4m3 and qscale [T], byte-
 * identical to ffb_attention followed by ffb_quantize_fp8 (FFB_QUANT_ROWWISE).  Replaces
 * `attention_direct` (_legacy/limit_kernels.py:36-45) plus `quantize_rows`
 * (_legacy/fp8_private.py:11-18) on the per-token-scale path.  Each row's maximum over its
 * HQ heads is combined across the CTAs of its 128-row query tile (per-head maxima in the
 * scratch, an arrival counter and a bounded wait), so every CTA of the grid,
 * ceil(T/128) * HQ, must be resident at once: FFB_EUNSUPPORTED when that exceeds the SM
 * count.  HQ a multiple of 4.  sync: ffb_attention_rowwise_sync_bytes(T, HQ) bytes, 16-byte
 * aligned, zero before the first call and not touched by the caller between calls (its
 * counters carry over from call to call; zero it again after a device error).  Calls
 * sharing one sync must run in stream order. */
int ffb_attention_rowwise(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint8_t* out8,
                          float* qscale, void* sync, int T, int HQ, int HK, float scale, void* stream);

/* Scratch bytes ffb_attention_rowwise needs for T rows and HQ heads (no reference
 * counterpart). */
int ffb_attention_rowwise_sync_bytes(int T, int HQ);

/* Copies rows index[i] of src [*, row_bytes] to dst [n, row_bytes] (index on device;
 * the tail's `h.index_select(1, pick)`, _family/night_runtime.py:103). */
int ffb_gather_rows(const void* src, const int64_t* index, void* dst, int n, int row_bytes,
                    void* stream);

/* Activation FP8 quantisation of a bf16 [M,K] matrix.
 * STATIC replaces _family/depth_fp8.py:8-19 (`_runtime_scale`); ROWWISE replaces
 * _legacy/fp8_private.py:11-18 (`quantize_rows`).  q8 [M,K]; qscale [M] (ROWWISE: written;
 * ROWSCALE: read, the quotient x / qscale[row] as ROWWISE forms it). */
int ffb_quantize_fp8(const uint16_t* x, int quant_mode, float inv_scale,
                     uint8_t* q8, float* qscale, int M, int K, void* stream);

/* Set-up-time weight quantisation W [N,K] bf16 -> W8 [N,K] e4m3 + fp32 scale.
 * per_channel = 0: one scale (_legacy/limit_kernels.py:122-127, StaticFP8Linear);
 * per_channel = 1: scale[N] (_legacy/fp8_private.py:22-27, FP8Linear).
 * ws: >= 4*N bytes of scratch. */
int ffb_quantize_weight_fp8(const uint16_t* w, int per_channel, uint8_t* w8, float* scale,
                            void* ws, int N, int K, void* stream);

/* ffb_quantize_weight_fp8 without caller scratch.  This entry point has no counterpart in
 * the reference.  The per-row maxima live in a fixed device array inside the library
 * (FFB_QW_NOALLOC_MAX_N fp32 entries, 256 KiB per device), so a caller that cannot
 * allocate device memory - a C host that owns only the weight and its outputs, or a
 * process already at its device-memory cap - can still quantise weights.
 *   - allocates nothing: no cudaMalloc/cudaFree and no allocating library call;
 *   - N > FFB_QW_NOALLOC_MAX_N is rejected with FFB_EINVAL (use ffb_quantize_weight_fp8);
 *   - the first call on each device looks the array up with cudaGetSymbolAddress, with
 *     that device current (this may load the library's device code); make that first
 *     call before any stream capture;
 *   - nothing in the array has to start at zero: a call writes every entry it reads;
 *   - one array per device, shared by every call on it: calls whose execution overlaps
 *     (different streams, different host threads) race on it; calls on one stream are
 *     ordered and safe;
 *   - `stream` must belong to the current device.
 * Arguments and results are those of ffb_quantize_weight_fp8 without `ws`. */
#define FFB_QW_NOALLOC_MAX_N 65536
int ffb_quantize_weight_fp8_noalloc(const uint16_t* w, int per_channel, uint8_t* w8, float* scale,
                                    int N, int K, void* stream);

/* FP8 e4m3 W8A8 GEMM on tcgen05 (kind::f8f6f4), fp32 accumulation in tensor memory.
 * Replaces _family/depth_fp8.py:22-26 (`RuntimeScaleLinear.__call__` -> torch._scaled_mm)
 * and _legacy/fp8_private.py:29-38.  a8 [M,K] activations, w8 [N,K] weights (K-major);
 * a_scale is [M] (a_per_row) or [1]; w_scale is [N] (w_per_col) or [1];
 * out = (a8 . w8^T) * a_scale[m] * w_scale[n].
 * epilogue FFB_EPI_BF16: out [M,N] bf16; FFB_EPI_F32_PARTIAL: ws [splits][M][N] fp32
 * (K split `splits` ways; the consumer sums the splits); FFB_EPI_SWIGLU: out [M,N/2] bf16
 * with w8 rows (and a per-channel w_scale) in ffb_pack_gateup order.
 * feature_tile: 128 or 256 output features per token-major tile (128 tokens x 128/256
 * features per MMA tile); FFB_TILE_STREAM: the weight-stationary schedule (weights on the
 * MMA's M side, each CTA one 128-feature weight tile (two, gate and up, for SwiGLU), a
 * range of at most 256 tokens and one of the `splits` K ranges; needs M <= 256 x CTAs per
 * tile and tiles x splits <= SMs); 0 = the weight-stationary schedule when splits == 1,
 * M <= 512 and it applies, else 256 when N allows, else 128.  Every choice gives the same
 * bytes for the same `splits`. */
#define FFB_TILE_STREAM 1
/* The number of CTAs ffb_fp8_gemm's weight-stationary schedule (FFB_TILE_STREAM) launches
 * for an M x N x K GEMM with this epilogue (FFB_EPI_BF16, FFB_EPI_F32_PARTIAL or
 * FFB_EPI_SWIGLU) and K split on the current device, or 0 when it does not apply.  A
 * host-side query (no device work) for planners; part of the same replacement as
 * ffb_fp8_gemm. */
int ffb_fp8_gemm_stream_ctas(int M, int N, int K, int epilogue, int splits);
int ffb_fp8_gemm(const uint8_t* a8, const float* a_scale, int a_per_row,
                 const uint8_t* w8, const float* w_scale, int w_per_col,
                 int epilogue, uint16_t* out, float* ws, int splits, int feature_tile,
                 int M, int N, int K, void* stream);

/* The qkv projection fused with per-head QK RMSNorm + interleaved-M-RoPE rotation.
 * Replaces the qkv `RuntimeScaleLinear` (_family/depth_fp8.py:22-26) followed by
 * `qk_pair` (_legacy/broad_kernels.py:63-74, rounding of lower_kernels.py:66-86): each
 * 128-feature tile is one head; its bf16 output row is normalised and rotated in the GEMM
 * epilogue.  w8 [(HQ+2HK)*128, K] packed q|k|v rows; q_norm/k_norm [128]; cos/sin [T,128]
 * rotate-half tables whose two 64-column halves are equal (cat(freqs, freqs), as every
 * Qwen3-VL / HF rotary table): only columns [0, 64) are read;
 * outputs head-major yq [HQ,T,128], yk [HK,T,128], yv [HK,T,128] (V unrotated). */
int ffb_fp8_gemm_qk_rope(const uint8_t* a8, const float* a_scale, int a_per_row,
                         const uint8_t* w8, const float* w_scale, int w_per_col,
                         const uint16_t* q_norm, const uint16_t* k_norm, float eps,
                         const uint16_t* cos, const uint16_t* sin,
                         uint16_t* yq, uint16_t* yk, uint16_t* yv,
                         int T, int HQ, int HK, int K, void* stream);

/* Producers fused into the front of an FP8 GEMM (ffb_fp8_gemm_fused,
 * ffb_fp8_gemm_qk_rope_fused).  The GEMM's CTAs first compute its FP8 activation operand
 * a8 (and the per-row scales) from bf16 rows, each CTA a slice of the M rows, then meet
 * at a bounded grid-wide barrier and run the GEMM on the rows just written: the pair
 * costs one launch instead of two, with results bit-identical to the separate calls. */
#define FFB_PRO_QUANT 1        /* a8 = ffb_quantize_fp8(x)                                         */
#define FFB_PRO_ADD_RMSNORM 2  /* a8 = the q8 output of ffb_add_rmsnorm(x, b | b32, deep, norm_w)  */

typedef struct ffb_gemm_prologue {
  int kind;                /* FFB_PRO_QUANT or FFB_PRO_ADD_RMSNORM                          */
  const uint16_t* x;       /* QUANT: bf16 [M,K] to quantise; ADD_RMSNORM: residual input a  */
  const uint16_t* b;       /* ADD_RMSNORM: bf16 addend [M,K], or NULL (then b32 / no add)   */
  const float* b32;        /* ADD_RMSNORM: fp32 split-K partials [splits][M][K] if b is NULL */
  int splits;              /* 1..8 partial tiles in b32                                     */
  int add;                 /* ADD_RMSNORM: 0 = plain RMSNorm of x (ffb_rmsnorm)             */
  const uint16_t* deep;    /* ADD_RMSNORM: deepstack rows [nv,K] added to [start, start+nv) */
  int start, nv;
  const uint16_t* norm_w;  /* ADD_RMSNORM: RMSNorm weight [K]                               */
  float eps;
  uint16_t* residual;      /* ADD_RMSNORM: bf16 residual rows out (may be NULL)             */
  int quant_mode;          /* FFB_QUANT_STATIC or FFB_QUANT_ROWWISE                         */
  float inv_scale;         /* STATIC: multiplier applied before the e4m3 cast               */
  uint64_t* sync;          /* one 8-byte device word, zero before the first call; one word
                              per stream (calls on different streams must not share it);
                              zero it again after a FFB_ETIMEOUT device error              */
} ffb_gemm_prologue;

/* ffb_fp8_gemm whose activation operand is produced by the fused prologue `pro`:
 * replaces ffb_quantize_fp8 (or ffb_add_rmsnorm / ffb_rmsnorm with FP8 output) followed by
 * ffb_fp8_gemm - in the reference, `quantize_rows` / `_runtime_scale`
 * (_legacy/fp8_private.py:11-18, _family/depth_fp8.py:8-12) or `add_rms`
 * (_legacy/lower_kernels.py:24-32) followed by the linear (_family/depth_fp8.py:22-26).
 * a8 [M,K] and a_scale ([M] when ROWWISE, written here; the per-tensor device scale when
 * STATIC, read) are the prologue's outputs and the GEMM's inputs; a_per_row must equal
 * (pro->quant_mode == FFB_QUANT_ROWWISE).  K must be a multiple of 8 and at most 36864
 * (QUANT) or 9216 (ADD_RMSNORM).  Other arguments as ffb_fp8_gemm. */
int ffb_fp8_gemm_fused(const ffb_gemm_prologue* pro, uint8_t* a8, float* a_scale, int a_per_row,
                       const uint8_t* w8, const float* w_scale, int w_per_col,
                       int epilogue, uint16_t* out, float* ws, int splits, int feature_tile,
                       int M, int N, int K, void* stream);

/* ffb_fp8_gemm_qk_rope with the fused prologue `pro` (as ffb_fp8_gemm_fused): replaces the
 * add_rms / rms_one of the layer input, its quantisation, and the qkv linear + qk_pair. */
int ffb_fp8_gemm_qk_rope_fused(const ffb_gemm_prologue* pro, uint8_t* a8, float* a_scale, int a_per_row,
                               const uint8_t* w8, const float* w_scale, int w_per_col,
                               const uint16_t* q_norm, const uint16_t* k_norm, float eps,
                               const uint16_t* cos, const uint16_t* sin,
                               uint16_t* yq, uint16_t* yk, uint16_t* yv,
                               int T, int HQ, int HK, int K, void* stream);

/* Gate/up GEMM with the SwiGLU epilogue followed by the STATIC FP8 quantisation of the down
 * projection's input, in one launch: out8[m,c] = e4m3(clamp(bf16(bf16(silu(g)) * u) * out_inv,
 * +-448)) (u8 [M, N/2]), byte-identical to FFB_EPI_SWIGLU followed by ffb_quantize_fp8
 * (FFB_QUANT_STATIC, out_inv).  Replaces `swiglu` (_legacy/search_kernels.py:18-23) plus the
 * down projection's `_runtime_scale` (_family/depth_fp8.py:8-12) on the static-scale path.
 * Operands and scales as ffb_fp8_gemm with the gate/up interleave of ffb_pack_gateup;
 * feature tile 256; out_inv > 0. */
int ffb_fp8_gemm_swiglu_fp8(const uint8_t* a8, const float* a_scale, int a_per_row,
                            const uint8_t* w8, const float* w_scale, int w_per_col, float out_inv,
                            uint8_t* out8, int M, int N, int K, void* stream);

/* Reorders the rows of a [2I,K] gate/up weight (gate rows 0..I-1, up rows I..2I-1) into
 * the FFB_EPI_SWIGLU tile order: tile t = gate rows 128t..128t+127 then up rows
 * 128t..128t+127 (I must be a multiple of 128).  Works on rows of `elem_bytes`*K bytes:
 * bf16 / e4m3 weights, or a per-channel fp32 scale vector with K = 1, elem_bytes = 4. */
int ffb_pack_gateup(const void* src, void* dst, int I, int K, int elem_bytes, void* stream);

/* SwiGLU on strided gate/up views: y[m,i] = bf16(bf16(g/(1+exp(-g))) * u).
 * Replaces _legacy/search_kernels.py:8-23 (`swiglu`).  gate/up rows have stride
 * `row_stride` elements; y is [M, I] contiguous. */
int ffb_swiglu(const uint16_t* gate, const uint16_t* up, int row_stride, uint16_t* y,
               int M, int I, void* stream);

/* Final tail readout: chosen = bf16(residual + mlp), final RMSNorm, dot with the n
 * option rows, then log-softmax over the first k.
 * Replaces _legacy/limit_kernels.py:48-66 (`lm_readout`) + the `residual[0] + mlp`
 * add of _family/night_runtime.py:104.  mlp is a bf16 row, or (mlp == NULL) the sum of
 * `splits` fp32 partial rows mlp32[splits][H] (rounded to bf16), or absent when both
 * are NULL.  logits [n] fp32 (bf16-rounded dots as in the reference), logprobs [k] fp32
 * (may be NULL). */
int ffb_readout(const uint16_t* residual, const uint16_t* mlp, const float* mlp32, int splits,
                const uint16_t* norm_w, float eps, const uint16_t* head, int n, int k,
                float* logits, float* logprobs, int H, void* stream);

/* Symmetric int4 group-128 weight packing for the W4A16 path:
 * s = bf16(max|W_g|/7), q = clamp(rne(W/s), -8, 7), two nibbles per byte along K
 * (low nibble = even k).  packed [N, K/2] uint8, scales [N, K/128] bf16.
 * Replaces the packing of _family/night_runtime.py:15-26 (`Int4.__init__`) with the
 * symmetric g128 scheme. */
int ffb_pack_int4(const uint16_t* w, uint8_t* packed, uint16_t* scales, int N, int K,
                  void* stream);

/* W4A16 GEMM: out[m,n] = bf16( sum_k x[m,k] * bf16(q[n,k] * s[n,k/128]) ), weights
 * dequantised to bf16 in shared memory and multiplied on tcgen05 (kind::f16).
 * Replaces _family/night_runtime.py:31-33 (`Int4.__call__` -> _weight_int4pack_mm).
 * x [M,K] bf16 (K a multiple of 128); packed/scales as written by ffb_pack_int4;
 * epilogue FFB_EPI_BF16 / FFB_EPI_F32_PARTIAL / FFB_EPI_SWIGLU as for ffb_fp8_gemm, without
 * scales (they are inside the dequantised weights); feature_tile 128 or 256 (0 = 256
 * when N allows; SwiGLU always 256). */
int ffb_w4a16_gemm(const uint16_t* x, const uint8_t* packed, const uint16_t* scales,
                   int epilogue, uint16_t* out, float* ws, int splits, int feature_tile,
                   int M, int N, int K, void* stream);

/* Input packing in front of the vision tower: RGB canvas -> patch rows.
 * Replaces _legacy/sub10_runtime.py:21-29 (`pack_rgb`, height == width) and
 * _family/depth_runtime.py:18-25 (`pack_rectangle`).  rgb [height, width, 3] u8 (HWC,
 * row-major, any alignment); pixels [(height/16)*(width/16), 1536] bf16, 16-byte aligned:
 * row p = patch p in 2x2 merge-group order, element c*512 + t*256 + y*16 + x =
 * bf16((rgb[y', x', c] - 127.5) / 127.5) for both temporal copies t.  height and width
 * must be positive multiples of 32 (at most 2^26 pixels). */
int ffb_pack_rgb(const uint8_t* rgb, uint16_t* pixels, int height, int width, void* stream);

/* ffb_pack_rgb over n canvases of one size in one launch (no reference counterpart: the
 * reference packs one canvas per request; batched prefill packs a batch at once).
 * rgb [n, height, width, 3] u8; pixels [n * (height/16)*(width/16), 1536] bf16, canvas i's
 * patch rows at rows [i*P, (i+1)*P); n * height * width <= 2^30. */
int ffb_pack_rgb_batch(const uint8_t* rgb, uint16_t* pixels, int n, int height, int width,
                       void* stream);

/* ---------------------------------------------------------------- tensor parallel, peer memory
 * One process per GPU.  The o_proj / down_proj partial sums and the per-token activation
 * maxima of the tensor-parallel ranks are read straight from each other's memory over
 * NVLink (CUDA IPC mappings; plain loads, stores and atomics, no multicast), by the kernel
 * that consumes them, instead of after an NCCL collective.  No reference counterpart (the
 * reference runs on one GPU, api.py:56-57). */

#define FFB_MAX_PEERS 8

/* Handshake state of one rank: flags[p] is rank p's [world][nslots] uint32 array (for
 * p == rank this process's own, else the IPC mapping of rank p's); local is this rank's
 * [nslots] uint32 call counts.  Both zero before the first call of any rank.  Slot i is
 * used by CTA i of a call; every rank must make the same sequence of calls. */
typedef struct ffb_peer_sync {
  uint32_t* flags[FFB_MAX_PEERS];
  uint32_t* local;
  int rank, world, nslots;
} ffb_peer_sync;

/* Device allocation of `bytes` (zeroed) with its 64-byte CUDA IPC handle, and the mapping
 * of another process's allocation from its handle (peer access enabled lazily). */
int ffb_peer_alloc(size_t bytes, void** dptr, void* handle);
int ffb_peer_open(const void* handle, void** dptr);
int ffb_peer_close(void* dptr);
int ffb_peer_free(void* dptr);

/* ffb_add_rmsnorm whose b is the sum of the ranks' fp32 partial planes: planes[r] (host
 * array of `world` device pointers; rank r's [T, H] plane, peer-mapped) are summed in rank
 * order ((p0 + p1) + p2 ...), then rounded to bf16 as the linear's output.  Replaces the
 * NCCL all-reduce of the row-parallel o_proj / down_proj partials plus the residual add +
 * RMSNorm (_legacy/lower_kernels.py:7-32) of a tensor-parallel layer.  A grid of at most four
 * CTAs per SM strides over the rows; CTA i handshakes slot i with every rank once before
 * reading the planes (its own rank's producer has finished by stream order); a wait that
 * gives up after 2 s sets the device error word.  Slots used: min(T, 4 x SMs). */
int ffb_add_rmsnorm_peers(const uint16_t* a, const float* const* planes, const ffb_peer_sync* sync,
                          const uint16_t* deep, int start, int nv, const uint16_t* w, float eps,
                          uint16_t* residual, uint16_t* out, int quant_mode, float inv_scale,
                          uint8_t* q8, float* qscale, int T, int H, void* stream);

/* ffb_quantize_fp8 (ROWWISE) of a row split over the tensor-parallel ranks (x is this
 * rank's [M, K] slice): each row's slice maximum is written into every rank's amax[p]
 * ([world][M] fp32, host array of device pointers), the ranks handshake the row's slot, and
 * the scale is max(max over ranks, 1e-12) / 448 -- the unsharded row's scale, as
 * ffb_quantize_fp8 ROWWISE + an all-reduce (MAX) of the scales + FFB_QUANT_ROWSCALE. */
int ffb_quantize_fp8_peers(const uint16_t* x, float* const* amax, const ffb_peer_sync* sync,
                           uint8_t* q8, float* qscale, int M, int K, void* stream);

/* ---------------------------------------------------------------- vision tower
 * The kernels of the Qwen3-VL vision tower in front of the language path (patch embedding,
 * ViT blocks, deepstack and final mergers).  The reference runs it as HF modules plus its
 * Triton vision RoPE (_legacy/vision_graph_runtime.py:16-27, `VisionGraph.core`;
 * scaled_qwen_runtime.py:42-55, `NativeNormVision.core`). */

/* bf16 linear on tcgen05 (kind::f16): out[m,n] = epilogue(sum_k a[m,k] * w[n,k] + bias[n]).
 * Replaces the blocks' and mergers' nn.Linear calls and the patch embedding's Conv3d (as a
 * [P, 1536] x [C, 1536]^T product); the epilogues fold in the residual add that follows
 * attn.proj / mlp.linear_fc2 (and the position embedding after the patch embedding), and the
 * GELU after linear_fc1 (tanh form in the blocks, erf form in the mergers; own polynomial
 * tanh and Abramowitz-Stegun 7.1.26 erf, within 5e-7 of the exact functions).
 * a [M,K], w [N,K] (K-major, as nn.Linear stores it), bias [N] or NULL, res [M,N]
 * (FFB_EPI_BIAS_RES, may alias out), out [M,N], all bf16 and 16-byte aligned; K and N
 * multiples of 8.  feature_tile 64 / 128 / 256 (0 = the plan's).  splits > 1 splits K, the
 * partial sums added in split order ((p0 + p1) + p2 ...) before the epilogue.  A 256-wide
 * tile split 2 or 4 ways runs as thread-block clusters (one CTA per split) that reduce over
 * distributed shared memory: ws and counters are not used and may be NULL.  Every other
 * split writes an fp32 partial plane to ws [splits][M][N] (16-byte aligned) and the split
 * that finishes last sums the planes and runs the epilogue; counters
 * [ceil(M/128) * ceil(N/feature_tile)] uint32 must be zero before the first call and are
 * left zero by every call that completes. */
int ffb_bf16_gemm(const uint16_t* a, const uint16_t* w, const uint16_t* bias, const uint16_t* res,
                  int epilogue, uint16_t* out, int feature_tile, int splits, float* ws,
                  uint32_t* counters, int M, int N, int K, void* stream);

/* The plan ffb_bf16_gemm uses for M x N x K on the current device: plan[0] = feature tile,
 * plan[1] = K splits, plan[2] = counters that plan needs (0 when it needs no ws / counters;
 * no reference counterpart; a host-side query). */
int ffb_bf16_gemm_plan(int M, int N, int K, int* plan);

/* LayerNorm over rows of C: y = bf16(((x - mean) * rstd) * w + b), mean and variance from
 * float64 sums, rstd = 1 / sqrt(var + eps).  Replaces the vision blocks' norm1 / norm2 and
 * the mergers' norm (nn.LayerNorm, _legacy/vision_graph_runtime.py:16-27; the add + LayerNorm
 * of _legacy/lower_kernels.py:115-136 with the add done by the producing linear).
 * x, y [rows, C], w, b [C] bf16, 16-byte aligned; C a multiple of 8, at most 8192. */
int ffb_layernorm(const uint16_t* x, const uint16_t* w, const uint16_t* b, float eps, uint16_t* y,
                  int rows, int C, void* stream);

/* Add + LayerNorm: residual = bf16(a + add), y = LayerNorm(residual) as ffb_layernorm.
 * Replaces `add_layernorm` (_legacy/lower_kernels.py:115-136).  With add == NULL it is
 * ffb_layernorm (residual unused).  a, add, residual, y [rows, C]; w, b [C]; bf16. */
int ffb_add_layernorm(const uint16_t* a, const uint16_t* add, const uint16_t* w, const uint16_t* b,
                      float eps, uint16_t* residual, uint16_t* y, int rows, int C, void* stream);

/* 2-D vision rotary on the qkv projection, and the head-major layout of the attention
 * kernel.  Replaces `_vision_rope` (_legacy/search_kernels.py:111-125): for q and k,
 * y[c] = x[c] * cos[c] + r[c] * sin[c] with r = rotate_half(x) (each product and the sum
 * rounded to fp32, then bf16).  qkv [P, 3*H*d] bf16 (patch rows [q | k | v], heads of d);
 * cos, sin [P, d] fp32; q, k, v [H, P, dp] bf16: columns [0, d) written, columns [d, dp)
 * left untouched (the attention's zero padding: zero them once) (dp >= d; d and dp
 * multiples of 8, H * d <= 7680; qkv, q, k, v, cos, sin 16-byte aligned). */
int ffb_vision_rope(const uint16_t* qkv, const float* cos, const float* sin, int P, int H, int d,
                    int dp, uint16_t* q, uint16_t* k, uint16_t* v, void* stream);

/* Non-causal multi-head attention over the T patches of one image (every query sees every
 * key), the arithmetic of ffb_attention otherwise.  Replaces the vision blocks' SDPA
 * (_legacy/vision_graph_runtime.py:16-27, one image per sequence).  q, k, v [H, T, 128]
 * bf16 with the head dimension d zero-padded to 128 (as ffb_vision_rope writes them with
 * dp = 128); out [T, H*d] bf16 (d a multiple of 8, at most 128). */
int ffb_attention_full(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
                       int T, int H, int d, float scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FFB200_H */
