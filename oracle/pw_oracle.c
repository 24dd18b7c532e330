/*
 * pw_oracle.c -- CPU restatement of Prismwing's block-FP8 routed-MoE semantics.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path: it
 * may be called by tests/, by __graft_entry__.smoke() and by bench.py's
 * cpu_baseline / --impl reference legs, and by nothing else.  The product
 * (the CUDA library behind include/pw_cuda.h) never links or calls it.
 *
 * Every function names the reference function it restates (path:line inside
 * the x3haloed/mimo-prismwing source tree).  Build with -ffp-contract=off so
 * that `a += b * c` rounds the product before the add, as Rust does.
 *
 * Two accumulation modes exist wherever a long sum appears:
 *   PWO_ACC_F32  -- the reference's own f32 order (sequential, no FMA);
 *   PWO_ACC_F64  -- every product and partial sum in f64, rounded to f32
 *                   once at the end (the parity tolerance is quoted against
 *                   this mode).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Thread count for the row-parallel loops (rows are independent, so the
 * result does not depend on it). */
void pwo_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int pwo_get_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

#define PWO_ACC_F32 0
#define PWO_ACC_F64 1

#define PWO_LAYOUT_PLAIN 0
#define PWO_LAYOUT_FULL_QKV 1
#define PWO_LAYOUT_SWA_QKV 2

float pwo_sleef_expf_u10(float d);
float pwo_sigmoid(float logit);
float pwo_staged_swiglu(float gate, float up, int exp_kind);

static inline uint32_t f2u(float v) { uint32_t u; memcpy(&u, &v, 4); return u; }
static inline float u2f(uint32_t u) { float v; memcpy(&v, &u, 4); return v; }

/* ------------------------------------------------------------------ */
/* e4m3fn decode: src/lib.rs:7456 (decode_f8_e4m3fn).                  */
/* Exponent 0 is subnormal (m/8 * 2^-6); 0x7f / 0xff are NaN with the  */
/* reference's payload 0x7ff00000 (sign kept); all else is normal.     */
/* ------------------------------------------------------------------ */
float pwo_decode_e4m3(uint8_t bits) {
  const float sign = (bits & 0x80) ? -1.0f : 1.0f;
  const int e = (bits >> 3) & 0x0f;
  const int m = bits & 0x07;
  if (e == 0) return sign * ldexpf((float)m / 8.0f, -6);
  if (e == 15 && m == 7) return u2f(((uint32_t)(bits & 0x80) << 24) | 0x7ff00000u);
  return sign * ldexpf(1.0f + (float)m / 8.0f, e - 7);
}

/* ------------------------------------------------------------------ */
/* f32 -> bf16 round-to-nearest-even kept in f32 storage:              */
/* src/text_endpoint.rs:2960 (round_bf16).  Infinities pass through;   */
/* NaNs become quiet with the upper 16 payload bits kept.              */
/* ------------------------------------------------------------------ */
float pwo_round_bf16(float value) {
  const uint32_t bits = f2u(value);
  if ((bits & 0x7f800000u) == 0x7f800000u) {
    if ((bits & 0x007fffffu) == 0) return value;
    const uint32_t payload = ((bits >> 16) & 0xffffu) | 0x0040u;
    return u2f(payload << 16);
  }
  const uint32_t bias = 0x7fffu + ((bits >> 16) & 1u);
  return u2f((bits + bias) & 0xffff0000u);
}

void pwo_round_bf16_array(const float *in, float *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = pwo_round_bf16(in[i]);
}

void pwo_decode_e4m3_array(const uint8_t *in, float *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = pwo_decode_e4m3(in[i]);
}

void pwo_sleef_expf_array(const float *in, float *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = pwo_sleef_expf_u10(in[i]);
}

void pwo_sigmoid_array(const float *in, float *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = pwo_sigmoid(in[i]);
}

void pwo_staged_swiglu_array(const float *gate, const float *up, float *out, size_t n, int exp_kind) {
  for (size_t i = 0; i < n; ++i) out[i] = pwo_staged_swiglu(gate[i], up[i], exp_kind);
}

/* ------------------------------------------------------------------ */
/* e4m3fn encode by nearest-value search over codes 0..0x7e with ties  */
/* to the even code: src/text_endpoint.rs:2985 (encode_f8_e4m3fn).     */
/* Returns -1 for a non-finite value or |value| > 448.                 */
/* ------------------------------------------------------------------ */
int pwo_encode_e4m3_search(float value, uint8_t *out) {
  if (!isfinite(value) || fabsf(value) > 448.0f) return -1;
  const uint8_t sign = signbit(value) ? 0x80 : 0x00;
  if (value == 0.0f) { *out = sign; return 0; }
  const float magnitude = fabsf(value);
  uint8_t best = 0;
  float best_distance = INFINITY;
  for (int candidate = 0; candidate <= 0x7e; ++candidate) {
    const float distance = fabsf(magnitude - pwo_decode_e4m3((uint8_t)candidate));
    if (distance < best_distance ||
        (distance == best_distance && (candidate & 1) == 0 && (best & 1) != 0)) {
      best = (uint8_t)candidate;
      best_distance = distance;
    }
  }
  *out = (uint8_t)(best | sign);
  return 0;
}

/* Same mapping computed by exact RNE arithmetic (no search).  Not in the
 * reference; tests use it to show the search equals IEEE round-to-nearest-
 * even into e4m3 (which is what the GPU's cvt.rn.satfinite does). */
int pwo_encode_e4m3_rne(float value, uint8_t *out) {
  if (!isfinite(value) || fabsf(value) > 448.0f) return -1;
  const uint8_t sign = signbit(value) ? 0x80 : 0x00;
  const double a = fabs((double)value);
  /* quantum: 2^-9 below 2^-6 (subnormal), else 2^(floor(log2 a) - 3) */
  double q;
  if (a < ldexp(1.0, -6)) {
    q = ldexp(1.0, -9);
  } else {
    int e;
    frexp(a, &e); /* a = f * 2^e, f in [0.5,1) -> floor(log2 a) = e-1 */
    q = ldexp(1.0, e - 1 - 3);
  }
  const double k = a / q; /* exact: q is a power of two */
  double r = floor(k);
  const double frac = k - r;
  if (frac > 0.5 || (frac == 0.5 && fmod(r, 2.0) != 0.0)) r += 1.0;
  const double rounded = r * q;
  /* find the code whose decode equals `rounded` */
  for (int c = 0; c <= 0x7e; ++c) {
    if ((double)pwo_decode_e4m3((uint8_t)c) == rounded) { *out = (uint8_t)(c | sign); return 0; }
  }
  return -2;
}

/* ------------------------------------------------------------------ */
/* Dynamic per-token, per-128-column FP8 activations:                  */
/* src/text_endpoint.rs:3008 (dynamic_fp8_activations).                */
/* scale = max(absmax, 1e-10) / 448; code = enc(clamp(x/scale,±448));  */
/* deq = dec(code) * scale.  Any of codes/scales/deq may be NULL.      */
/* ------------------------------------------------------------------ */
int pwo_dynamic_fp8(const float *input, size_t rows, size_t columns, uint8_t *codes,
                    float *scales, float *dequantized) {
  const size_t group = 128;
  if (rows == 0 || columns == 0 || columns % group != 0) return -1;
  for (size_t i = 0; i < rows * columns; ++i)
    if (!isfinite(input[i])) return -1;
  const size_t groups = columns / group;
  for (size_t r = 0; r < rows; ++r) {
    for (size_t g = 0; g < groups; ++g) {
      const float *src = input + r * columns + g * group;
      float absmax = 0.0f;
      for (size_t i = 0; i < group; ++i) absmax = fmaxf(absmax, fabsf(src[i]));
      absmax = fmaxf(absmax, 1.0e-10f);
      const float scale = absmax / 448.0f;
      if (!isfinite(scale) || scale <= 0.0f) return -2;
      if (scales) scales[r * groups + g] = scale;
      for (size_t i = 0; i < group; ++i) {
        float normalized = src[i] / scale;
        if (normalized < -448.0f) normalized = -448.0f;
        if (normalized > 448.0f) normalized = 448.0f;
        uint8_t code;
        if (pwo_encode_e4m3_search(normalized, &code) != 0) return -3;
        if (codes) codes[r * columns + g * group + i] = code;
        if (dequantized) dequantized[r * columns + g * group + i] = pwo_decode_e4m3(code) * scale;
      }
    }
  }
  return 0;
}

/* ------------------------------------------------------------------ */
/* Weight/scale view validation: src/lib.rs:1217                      */
/* (validate_fp8_views_internal).  Returns 0 or a negative code:       */
/*  -1 dims not nonzero multiples of 128, -2 input length/finiteness,  */
/*  -3 scale grid non-finite, -4 weight byte 0x7f/0xff (offset in *at). */
/* ------------------------------------------------------------------ */
int pwo_validate_fp8(const uint8_t *weight, const float *scale, size_t rows, size_t columns,
                     const float *input, size_t input_len, int scan_weights, size_t *at) {
  if (rows == 0 || columns == 0 || rows % 128 || columns % 128) return -1;
  if (input) {
    if (input_len != columns) return -2;
    for (size_t i = 0; i < input_len; ++i)
      if (!isfinite(input[i])) return -2;
  }
  for (size_t i = 0; i < (rows / 128) * (columns / 128); ++i)
    if (!isfinite(scale[i])) return -3;
  if (scan_weights) {
    for (size_t i = 0; i < rows * columns; ++i) {
      if (weight[i] == 0x7f || weight[i] == 0xff) {
        if (at) *at = i;
        return -4;
      }
    }
  }
  return 0;
}

/* ------------------------------------------------------------------ */
/* Readable block-FP8 GEMV, activation NOT quantized:                  */
/* src/lib.rs:1272 (mapped_fp8_gemv) and src/lib.rs:7469               */
/* (block_fp8_gemv).  y[r] = sum_c dec(W[r,c]) * S[r/128, c/128] * x[c] */
/* F32 mode: `sum += (dec*scale)*x` sequentially in c, no contraction. */
/* ------------------------------------------------------------------ */
int pwo_readable_gemv(const uint8_t *weight, const float *scale, size_t rows, size_t columns,
                      const float *input, float *output, int mode) {
  if (rows == 0 || columns == 0 || rows % 128 || columns % 128) return -1;
  const size_t scale_columns = columns / 128;
  int status = 0;
#pragma omp parallel for schedule(static) reduction(min : status)
  for (size_t r = 0; r < rows; ++r) {
    const uint8_t *row = weight + r * columns;
    const float *srow = scale + (r / 128) * scale_columns;
    if (mode == PWO_ACC_F32) {
      float sum = 0.0f;
      for (size_t c = 0; c < columns; ++c) {
        const float decoded = pwo_decode_e4m3(row[c]);
        if (!isfinite(decoded)) status = -4;
        const float scaled = decoded * srow[c / 128];
        const float term = scaled * input[c];
        sum += term;
      }
      output[r] = sum;
    } else {
      double sum = 0.0;
      for (size_t c = 0; c < columns; ++c) {
        const double decoded = (double)pwo_decode_e4m3(row[c]);
        if (!isfinite(decoded)) status = -4;
        sum += decoded * (double)srow[c / 128] * (double)input[c];
      }
      output[r] = (float)sum;
    }
    if (!isfinite(output[r]) && status == 0) status = -5;
  }
  return status;
}

/* ------------------------------------------------------------------ */
/* Fused QKV row maps: src/text_endpoint.rs:3174 (full_qkv_source_row),*/
/* :3200 (swa_qkv_source_row), :3227 (full_qkv_scale_row).            */
/* The checkpoint holds 4 tensor-parallel shards; logical rows are the */
/* global Q, then K, then V order.  Return (size_t)-1 out of range.     */
/* ------------------------------------------------------------------ */
enum { PWO_HEADS = 64, PWO_QK_HEAD = 192, PWO_V_HEAD = 128 };

size_t pwo_full_qkv_source_row(size_t logical) {
  const size_t q_rows = PWO_HEADS * PWO_QK_HEAD;   /* 12288 */
  const size_t k_rows = 4 * PWO_QK_HEAD;           /* 768 */
  const size_t v_rows = 4 * PWO_V_HEAD;            /* 512 */
  const size_t q_per_shard = q_rows / 4;           /* 3072 */
  const size_t shard_rows = q_per_shard + PWO_QK_HEAD + PWO_V_HEAD; /* 3392 */
  if (logical < q_rows) return (logical / q_per_shard) * shard_rows + logical % q_per_shard;
  if (logical < q_rows + k_rows) {
    const size_t local = logical - q_rows;
    return (local / PWO_QK_HEAD) * shard_rows + q_per_shard + local % PWO_QK_HEAD;
  }
  if (logical < q_rows + k_rows + v_rows) {
    const size_t local = logical - q_rows - k_rows;
    return (local / PWO_V_HEAD) * shard_rows + q_per_shard + PWO_QK_HEAD + local % PWO_V_HEAD;
  }
  return (size_t)-1;
}

size_t pwo_swa_qkv_source_row(size_t logical) {
  const size_t q_rows = PWO_HEADS * PWO_QK_HEAD;   /* 12288 */
  const size_t k_rows = 8 * PWO_QK_HEAD;           /* 1536 */
  const size_t v_rows = 8 * PWO_V_HEAD;            /* 1024 */
  const size_t qs = q_rows / 4, ks = k_rows / 4, vs = v_rows / 4;
  const size_t shard_rows = qs + ks + vs;          /* 3712 */
  if (logical < q_rows) return logical / qs * shard_rows + logical % qs;
  if (logical < q_rows + k_rows) {
    const size_t local = logical - q_rows;
    return local / ks * shard_rows + qs + local % ks;
  }
  if (logical < q_rows + k_rows + v_rows) {
    const size_t local = logical - q_rows - k_rows;
    return local / vs * shard_rows + qs + ks + local % vs;
  }
  return (size_t)-1;
}

size_t pwo_full_qkv_scale_row(size_t logical) {
  const size_t source = pwo_full_qkv_source_row(logical);
  if (source == (size_t)-1) return (size_t)-1;
  const size_t shard = source / 3392, local = source % 3392;
  size_t local_scale;
  if (local < 3072) local_scale = local / 128;
  else if (local < 3072 + PWO_QK_HEAD) local_scale = 24 + (local - 3072) / 128;
  else local_scale = 26;
  return shard * 27 + local_scale;
}

/* (source row, scale row) for a logical output row under a layout. */
static int layout_rows(int layout, size_t rows, size_t logical, size_t *source, size_t *scale_row) {
  if (layout == PWO_LAYOUT_PLAIN) {
    *source = logical;
    *scale_row = logical / 128;
    return 0;
  }
  if (layout == PWO_LAYOUT_FULL_QKV) {
    if (rows != 13568) return -1;
    *source = pwo_full_qkv_source_row(logical);
    *scale_row = pwo_full_qkv_scale_row(logical);
    return *source == (size_t)-1 ? -1 : 0;
  }
  if (layout == PWO_LAYOUT_SWA_QKV) {
    if (rows != 14848) return -1;
    *source = pwo_swa_qkv_source_row(logical);
    *scale_row = *source / 128;
    return *source == (size_t)-1 ? -1 : 0;
  }
  return -1;
}

/* ------------------------------------------------------------------ */
/* Block-scaled projection (SGLang operands):                           */
/* y[t,r] = sum_kb ( sum_{c in kb} dec(W[src(r),c]) * dec(code[t,c]) )  */
/*          * S[srow(r), kb] * xs[t, kb]                                */
/* src/wide_metal_moe.rs:404-423 (the CPU equation of                   */
/* probe_sglang_blockscaled_projection) and kernels/block_fp8_gemv.metal*/
/* :935-1046.  F32 mode: per block `dot += w*x` in increasing column,   */
/* then `total += dot*ws*xs` in increasing block.  F64 mode: all in     */
/* f64.  Output is the f32 pre-round value; `out` is [width, rows].     */
/* scale_columns is columns/128; scale row stride is scale_columns.     */
/* ------------------------------------------------------------------ */
int pwo_blockscaled_linear(const uint8_t *weight, const float *scale, size_t rows,
                           size_t columns, int layout, const uint8_t *codes,
                           const float *code_scales, size_t width, float *out, int mode) {
  if (rows == 0 || columns == 0 || columns % 128 || width == 0) return -1;
  const size_t blocks = columns / 128;
  float dec_lut[256];
  for (int i = 0; i < 256; ++i) dec_lut[i] = pwo_decode_e4m3((uint8_t)i);
  int status = 0;
#pragma omp parallel for schedule(static) reduction(min : status)
  for (size_t r = 0; r < rows; ++r) {
    size_t src, srow;
    if (layout_rows(layout, rows, r, &src, &srow) != 0) { status = -2; continue; }
    const uint8_t *wrow = weight + src * columns;
    const float *sv = scale + srow * blocks;
    for (size_t t = 0; t < width; ++t) {
      const uint8_t *xrow = codes + t * columns;
      const float *xsv = code_scales + t * blocks;
      if (mode == PWO_ACC_F32) {
        float total = 0.0f;
        for (size_t b = 0; b < blocks; ++b) {
          float dot = 0.0f;
          for (size_t i = 0; i < 128; ++i) {
            const float p = dec_lut[wrow[b * 128 + i]] * dec_lut[xrow[b * 128 + i]];
            dot += p;
          }
          const float a = dot * sv[b];
          const float term = a * xsv[b];
          total += term;
        }
        out[t * rows + r] = total;
      } else {
        double total = 0.0;
        for (size_t b = 0; b < blocks; ++b) {
          double dot = 0.0;
          for (size_t i = 0; i < 128; ++i)
            dot += (double)dec_lut[wrow[b * 128 + i]] * (double)dec_lut[xrow[b * 128 + i]];
          total += dot * (double)sv[b] * (double)xsv[b];
        }
        out[t * rows + r] = (float)total;
      }
    }
  }
  return status;
}

/* ------------------------------------------------------------------ */
/* SLEEF expf_u10 and the PyTorch-vectorised sigmoid:                  */
/* src/text_endpoint.rs:4511 (sleef_expf_u10), :4538                   */
/* (pytorch_sigmoid_f32).  The polynomial and Cody-Waite split are     */
/* SLEEF's published expf_u10 method; every multiply-add is a true FMA.*/
/* ------------------------------------------------------------------ */
float pwo_sleef_expf_u10(float d) {
  if (d < -104.0f) return 0.0f;
  if (d > 100.0f) return INFINITY;
  const float qf = nearbyintf(d * 1.442695040888963407359924681001892137f); /* RNE */
  const int q = (int)qf;
  float s = fmaf(qf, -0.693145751953125f, d);
  s = fmaf(qf, -1.428606765330187045e-06f, s);
  float u = 0.000198527617612853646278381f;
  u = fmaf(u, s, 0.00139304355252534151077271f);
  u = fmaf(u, s, 0.00833336077630519866943359f);
  u = fmaf(u, s, 0.0416664853692054748535156f);
  u = fmaf(u, s, 0.166666671633720397949219f);
  u = fmaf(u, s, 0.5f);
  u = fmaf(s * s, u, s) + 1.0f;
  const int q1 = q >> 1;
  const int q2 = q - q1;
  return (u * u2f((uint32_t)(q1 + 127) << 23)) * u2f((uint32_t)(q2 + 127) << 23);
}

float pwo_sigmoid(float logit) { return 1.0f / (1.0f + pwo_sleef_expf_u10(-logit)); }

/* ------------------------------------------------------------------ */
/* Staged bf16 SwiGLU: src/text_endpoint.rs:5336-5342 and              */
/* kernels/block_fp8_gemv.metal:139 (bf16_staged_swiglu):               */
/*   g = bf16(g); u = bf16(u); h = bf16( bf16(g / (1 + exp(-g))) * u ).  */
/* exp_kind 0 uses SLEEF expf_u10 (what the CUDA path uses), 1 uses the */
/* C library expf (what the reference's Rust CPU path calls).           */
/* ------------------------------------------------------------------ */
float pwo_staged_swiglu(float gate, float up, int exp_kind) {
  const float g = pwo_round_bf16(gate);
  const float u = pwo_round_bf16(up);
  const float e = exp_kind == 0 ? pwo_sleef_expf_u10(-g) : expf(-g);
  const float silu = pwo_round_bf16(g / (1.0f + e));
  return pwo_round_bf16(silu * u);
}

/* ------------------------------------------------------------------ */
/* Router logits, f32 accumulation in a fixed order.  The reference    */
/* computes f32 logits with an SGEMM (src/text_endpoint.rs:4350 via    */
/* f32_linear :3458) whose order is unspecified; this build pins the   */
/* order so that CPU and GPU agree bit for bit:                         */
/*   the K axis is cut into 256-column slices; slice s's sum is a chain */
/*   of fused multiply-adds in f32 (fmaf: one rounding per step) from   */
/*   +0 over its columns in ascending order; the logit is the slice    */
/*   sums added in slice order starting from slice 0's.  The weight is  */
/*   the checkpoint's F32 gate.weight (src/text_endpoint.rs:4350-4358)  */
/*   or bf16 bits (exact in f32); the chain is the same for both.       */
/* ------------------------------------------------------------------ */
static inline float bf16_bits_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

static int router_logits_any(const float *x, size_t tokens, const float *w32, const uint16_t *w16,
                             size_t experts, size_t hidden, float *logits) {
  if (hidden % 512 != 0) return -1;
  const size_t slices = hidden / 256;
#pragma omp parallel for schedule(static)
  for (size_t te = 0; te < tokens * experts; ++te) {
    const size_t t = te / experts, e = te % experts;
    const float *xr = x + t * hidden;
    float logit = 0.0f;
    for (size_t s = 0; s < slices; ++s) {
      float c = 0.0f;
      for (size_t i = 256 * s; i < 256 * (s + 1); ++i) {
        const float wv = w32 ? w32[e * hidden + i] : bf16_bits_to_f32(w16[e * hidden + i]);
        c = fmaf(xr[i], wv, c);
      }
      logit = s == 0 ? c : logit + c;
    }
    logits[t * experts + e] = logit;
  }
  return 0;
}

int pwo_router_logits(const float *x, size_t tokens, const uint16_t *weight_bf16, size_t experts,
                      size_t hidden, float *logits) {
  return router_logits_any(x, tokens, NULL, weight_bf16, experts, hidden, logits);
}

int pwo_router_logits_f32(const float *x, size_t tokens, const float *weight, size_t experts, size_t hidden,
                          float *logits) {
  return router_logits_any(x, tokens, weight, NULL, experts, hidden, logits);
}

/* ------------------------------------------------------------------ */
/* Sigmoid no-aux top-k routing.                                        */
/* Scores: sigmoid(logit) (src/text_endpoint.rs:4366).  Selection: top-k*/
/* of score+bias (src/text_endpoint.rs:4394 pytorch_noaux_routes).  The */
/* reference's std::nth_element order is platform-specific, so the      */
/* order emitted here is canonical: corrected score descending, index   */
/* ascending on ties (src/lib.rs:672-678).  Weights: score / (pairwise  */
/* sum of the eight chosen scores in that order + 1e-20)                */
/* (src/text_endpoint.rs:4382 pytorch_sum_eight).                       */
/* Returns number of rows whose k-th and (k+1)-th corrected scores tie  */
/* (>= 0), or a negative error.  margin[t] = kth - (k+1)th.             */
/* ------------------------------------------------------------------ */
static float sum_eight(const float v[8]) {
  const float lanes[4] = {v[0] + v[4], v[1] + v[5], v[2] + v[6], v[3] + v[7]};
  float s = 0.0f;
  for (int i = 0; i < 4; ++i) s += lanes[i];
  return s;
}

int pwo_noaux_topk(const float *logits, const float *bias, size_t tokens, size_t experts,
                   size_t top_k, uint32_t *selected, float *weights, float *scores_out,
                   float *margin) {
  if (top_k != 8 || experts <= top_k || experts > 4096) return -1;
  int ties = 0;
  float *scores = (float *)malloc(experts * sizeof(float));
  float *corrected = (float *)malloc(experts * sizeof(float));
  unsigned char *taken = (unsigned char *)malloc(experts);
  for (size_t t = 0; t < tokens; ++t) {
    for (size_t e = 0; e < experts; ++e) {
      if (!isfinite(logits[t * experts + e]) || !isfinite(bias[e])) { ties = -2; goto done; }
      scores[e] = pwo_sigmoid(logits[t * experts + e]);
      corrected[e] = scores[e] + bias[e];
      taken[e] = 0;
      if (scores_out) scores_out[t * experts + e] = scores[e];
    }
    uint32_t chosen[8];
    for (size_t k = 0; k < top_k + 1; ++k) {
      size_t best = experts;
      for (size_t e = 0; e < experts; ++e) {
        if (taken[e]) continue;
        if (best == experts || corrected[e] > corrected[best]) best = e;
      }
      if (k < top_k) { chosen[k] = (uint32_t)best; taken[best] = 1; }
      else {
        const float m = corrected[chosen[top_k - 1]] - corrected[best];
        if (margin) margin[t] = m;
        if (corrected[chosen[top_k - 1]] == corrected[best]) ties++;
      }
    }
    float chosen_scores[8];
    for (size_t k = 0; k < 8; ++k) chosen_scores[k] = scores[chosen[k]];
    const float denominator = sum_eight(chosen_scores) + 1.0e-20f;
    float wsum = 0.0f;
    for (size_t k = 0; k < 8; ++k) {
      selected[t * 8 + k] = chosen[k];
      weights[t * 8 + k] = chosen_scores[k] / denominator;
      wsum += weights[t * 8 + k];
    }
    if (fabsf(wsum - 1.0f) > 1.0e-6f) { ties = -3; goto done; }
  }
done:
  free(scores);
  free(corrected);
  free(taken);
  return ties;
}

/* ------------------------------------------------------------------ */
/* Routed MoE layer: src/text_endpoint.rs:5290 (routed_mlp_traced) with */
/* the wide runtime's staging (src/wide_metal_moe.rs:1081-1270):        */
/*  schedule expert -> [(position, weight)] in ascending expert, then   */
/*  ascending position; per expert: quantize gathered rows, gate and up */
/*  block-scaled projections, staged bf16 SwiGLU, quantize hidden, down */
/*  projection, bf16 round; out[pos] += bf16(down) * w in ascending     */
/*  expert order (product rounded, then added); final bf16 round.        */
/* Weights are per-expert pointers (experts[e*6 + {0..5}] = gate_w,     */
/* gate_s, up_w, up_s, down_w, down_s as void*).                         */
/* down_out (optional) receives bf16(down) per placement in schedule    */
/* order, [placements, hidden].                                          */
/* ------------------------------------------------------------------ */
int pwo_routed_layer(const float *input, size_t tokens, size_t hidden, size_t intermediate,
                     const uint32_t *selected, const float *route_weights, size_t experts,
                     const void *const *bank, int mode, int exp_kind, float *output,
                     float *hidden_out, float *down_out) {
  if (tokens == 0 || hidden % 128 || intermediate % 128) return -1;
  const size_t placements = tokens * 8;
  /* counting sort by expert, stable in (position, slot) */
  size_t *count = (size_t *)calloc(experts + 1, sizeof(size_t));
  for (size_t p = 0; p < placements; ++p) {
    if (selected[p] >= experts) { free(count); return -2; }
    count[selected[p] + 1]++;
  }
  for (size_t e = 0; e < experts; ++e) count[e + 1] += count[e];
  size_t *order = (size_t *)malloc(placements * sizeof(size_t));
  size_t *fill = (size_t *)malloc(experts * sizeof(size_t));
  for (size_t e = 0; e < experts; ++e) fill[e] = count[e];
  for (size_t p = 0; p < placements; ++p) order[fill[selected[p]]++] = p;

  memset(output, 0, tokens * hidden * sizeof(float));
  int status = 0;
  float *gathered = (float *)malloc(tokens * hidden * sizeof(float));
  uint8_t *xcodes = (uint8_t *)malloc(tokens * hidden);
  float *xscales = (float *)malloc(tokens * (hidden / 128) * sizeof(float));
  float *gate = (float *)malloc(tokens * intermediate * sizeof(float));
  float *up = (float *)malloc(tokens * intermediate * sizeof(float));
  float *act = (float *)malloc(tokens * intermediate * sizeof(float));
  uint8_t *hcodes = (uint8_t *)malloc(tokens * intermediate);
  float *hscales = (float *)malloc(tokens * (intermediate / 128) * sizeof(float));
  float *down = (float *)malloc(tokens * hidden * sizeof(float));
  for (size_t e = 0; e < experts && status == 0; ++e) {
    const size_t begin = count[e], n = count[e + 1] - count[e];
    if (n == 0) continue;
    for (size_t i = 0; i < n; ++i) {
      const size_t pos = order[begin + i] / 8;
      memcpy(gathered + i * hidden, input + pos * hidden, hidden * sizeof(float));
    }
    const uint8_t *gw = (const uint8_t *)bank[e * 6 + 0];
    const float *gs = (const float *)bank[e * 6 + 1];
    const uint8_t *uw = (const uint8_t *)bank[e * 6 + 2];
    const float *us = (const float *)bank[e * 6 + 3];
    const uint8_t *dw = (const uint8_t *)bank[e * 6 + 4];
    const float *ds = (const float *)bank[e * 6 + 5];
    if (pwo_dynamic_fp8(gathered, n, hidden, xcodes, xscales, NULL) != 0) { status = -3; break; }
    pwo_blockscaled_linear(gw, gs, intermediate, hidden, PWO_LAYOUT_PLAIN, xcodes, xscales, n, gate, mode);
    pwo_blockscaled_linear(uw, us, intermediate, hidden, PWO_LAYOUT_PLAIN, xcodes, xscales, n, up, mode);
    for (size_t i = 0; i < n * intermediate; ++i) {
      act[i] = pwo_staged_swiglu(gate[i], up[i], exp_kind);
      if (!isfinite(act[i])) status = -4;
    }
    if (hidden_out)
      for (size_t i = 0; i < n; ++i)
        memcpy(hidden_out + (begin + i) * intermediate, act + i * intermediate, intermediate * sizeof(float));
    if (status) break;
    if (pwo_dynamic_fp8(act, n, intermediate, hcodes, hscales, NULL) != 0) { status = -3; break; }
    pwo_blockscaled_linear(dw, ds, hidden, intermediate, PWO_LAYOUT_PLAIN, hcodes, hscales, n, down, mode);
    for (size_t i = 0; i < n; ++i) {
      const size_t p = order[begin + i];
      const size_t pos = p / 8;
      const float w = route_weights[p];
      for (size_t c = 0; c < hidden; ++c) {
        const float y = pwo_round_bf16(down[i * hidden + c]);
        if (down_out) down_out[(begin + i) * hidden + c] = y;
        const float term = y * w;
        output[pos * hidden + c] += term;
      }
    }
  }
  for (size_t i = 0; i < tokens * hidden; ++i) {
    output[i] = pwo_round_bf16(output[i]);
    if (status == 0 && !isfinite(output[i])) status = -5;
  }
  free(count); free(order); free(fill); free(gathered); free(xcodes); free(xscales);
  free(gate); free(up); free(act); free(hcodes); free(hscales); free(down);
  return status;
}

/* Schedule only (ascending expert, ascending position) -- the order the
 * layer above and the GPU runtime use for placements.  order[i] is the
 * flat (token*8 + slot) index of placement i; offsets has experts+1
 * entries. */
int pwo_schedule(const uint32_t *selected, size_t tokens, size_t experts, uint32_t *offsets,
                 uint32_t *order) {
  const size_t placements = tokens * 8;
  memset(offsets, 0, (experts + 1) * sizeof(uint32_t));
  for (size_t p = 0; p < placements; ++p) {
    if (selected[p] >= experts) return -2;
    offsets[selected[p] + 1]++;
  }
  for (size_t e = 0; e < experts; ++e) offsets[e + 1] += offsets[e];
  uint32_t *fill = (uint32_t *)malloc(experts * sizeof(uint32_t));
  memcpy(fill, offsets, experts * sizeof(uint32_t));
  for (size_t p = 0; p < placements; ++p) order[fill[selected[p]]++] = (uint32_t)p;
  free(fill);
  return 0;
}

/* ------------------------------------------------------------------ */
/* RMSNorm (src/text_endpoint.rs:2939 rms_norm, with stable_rms_inverse */
/* src/lib.rs:1890 and its sum of squares                               */
/* pytorch_contiguous_inner_square_sum_f32 src/lib.rs:1905).  The sum  */
/* runs in PyTorch's vectorised cascade order: 4 lanes x 4 interleaved  */
/* registers x 4 levels of f32 accumulators; level 0 takes              */
/* 2^level_power steps of 16 squares, then each level is added into the */
/* next (and cleared) until the step count is not a multiple of that   */
/* level's span; leftovers go to level 0, levels fold into level 0,     */
/* registers into register 0, and lanes into the scalar tail's sum.     */
/* Products and sums round separately (no fused multiply-add).          */
/* ------------------------------------------------------------------ */
float pwo_rms_square_sum(const float *values, size_t n) {
  enum { LANES = 4, INTERLEAVE = 4, LEVELS = 4 };
  const size_t vector_count = n / LANES;
  const size_t cascade_size = vector_count / INTERLEAVE;
  size_t ceil_log2 = 0;
  if (cascade_size > 1) {
    size_t v = cascade_size - 1;
    while (v) { ++ceil_log2; v >>= 1; }
  }
  const size_t level_power = ceil_log2 / LEVELS > 4 ? ceil_log2 / LEVELS : 4;
  const size_t level_step = (size_t)1 << level_power;
  const size_t level_mask = level_step - 1;
  float acc[LEVELS][INTERLEAVE][LANES];
  memset(acc, 0, sizeof acc);
  size_t index = 0;
  while (index + level_step <= cascade_size) {
    for (size_t s = 0; s < level_step; ++s) {
      for (int r = 0; r < INTERLEAVE; ++r) {
        const size_t base = (index * INTERLEAVE + r) * LANES;
        for (int l = 0; l < LANES; ++l) {
          const float sq = values[base + l] * values[base + l];
          acc[0][r][l] += sq;
        }
      }
      ++index;
    }
    for (int level = 1; level < LEVELS; ++level) {
      for (int r = 0; r < INTERLEAVE; ++r)
        for (int l = 0; l < LANES; ++l) {
          acc[level][r][l] += acc[level - 1][r][l];
          acc[level - 1][r][l] = 0.0f;
        }
      if (index & (level_mask << (level * level_power))) break;
    }
  }
  while (index < cascade_size) {
    for (int r = 0; r < INTERLEAVE; ++r) {
      const size_t base = (index * INTERLEAVE + r) * LANES;
      for (int l = 0; l < LANES; ++l) {
        const float sq = values[base + l] * values[base + l];
        acc[0][r][l] += sq;
      }
    }
    ++index;
  }
  for (int level = 1; level < LEVELS; ++level)
    for (int r = 0; r < INTERLEAVE; ++r)
      for (int l = 0; l < LANES; ++l) acc[0][r][l] += acc[level][r][l];
  for (size_t vec = cascade_size * INTERLEAVE; vec < vector_count; ++vec)
    for (int l = 0; l < LANES; ++l) {
      const float v = values[vec * LANES + l];
      const float sq = v * v;
      acc[0][0][l] += sq;
    }
  for (int r = 1; r < INTERLEAVE; ++r)
    for (int l = 0; l < LANES; ++l) acc[0][0][l] += acc[0][r][l];
  float result = 0.0f;
  for (size_t i = vector_count * LANES; i < n; ++i) {
    const float sq = values[i] * values[i];
    result += sq;
  }
  for (int l = 0; l < LANES; ++l) result += acc[0][0][l];
  return result;
}

/* stable_rms_inverse (src/lib.rs:1890): 1 / sqrt(sum/n + eps); -1 on   */
/* empty or non-finite input or a non-positive / non-finite epsilon.    */
int pwo_rms_inverse(const float *values, size_t n, float epsilon, float *inverse) {
  if (n == 0 || !isfinite(epsilon) || epsilon <= 0.0f) return -1;
  for (size_t i = 0; i < n; ++i)
    if (!isfinite(values[i])) return -1;
  const float variance = pwo_rms_square_sum(values, n) / (float)n;
  *inverse = 1.0f / sqrtf(variance + epsilon);
  return 0;
}

/* rms_norm (src/text_endpoint.rs:2939): per row, out = bf16(bf16(x*inv) */
/* * weight[c]); inverse (optional) receives each row's inverse.         */
int pwo_rms_norm(const float *x, size_t rows, size_t cols, const float *weight, float epsilon, float *out,
                 float *inverse) {
  for (size_t r = 0; r < rows; ++r) {
    float inv;
    if (pwo_rms_inverse(x + r * cols, cols, epsilon, &inv) != 0) return -1;
    if (inverse) inverse[r] = inv;
    for (size_t c = 0; c < cols; ++c) {
      const float normalized = pwo_round_bf16(x[r * cols + c] * inv);
      out[r * cols + c] = pwo_round_bf16(normalized * weight[c]);
    }
  }
  return 0;
}

/* Residual add of the decoder layer (src/text_endpoint.rs:5576-5580): */
/* out = bf16(residual + projected).                                    */
void pwo_residual_add(const float *residual, const float *projected, size_t n, float *out) {
  for (size_t i = 0; i < n; ++i) out[i] = pwo_round_bf16(residual[i] + projected[i]);
}
