/*
 * rocket_oracle.c — CPU restatement of burn-rocket's reference arithmetic for
 * the offloaded path. TEST INFRASTRUCTURE ONLY: the parity tests, the smoke
 * check and bench.py's CPU-baseline leg call it as the checker; nothing in
 * the product (librocket_b200.so, burn_rocket_b200/) links or calls it.
 *
 * Every function names the reference file:line it restates (paths relative to
 * the royalcat/burn-rocket tree). Parity pins: the golden vectors of the
 * reference's own tests, reproduced in tests/test_oracle_golden.py.
 *
 * Built by oracle/Makefile into oracle/liboracle.so (OpenMP for the timed
 * CPU-baseline kernels).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ f16 */
/* IEEE binary16 conversions with round-to-nearest-even, as the `half` crate
 * (2.7.1) does for f16::from_f32 / to_f32 (used at ext.rs:2144-2170). */
uint16_t orc_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xff) { /* inf / nan */
    if (man) return (uint16_t)(sign | 0x7e00u | (man >> 13));
    return (uint16_t)(sign | 0x7c00u);
  }
  int32_t e = (int32_t)exp - 127 + 15;
  if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u); /* overflow -> inf */
  if (e <= 0) {                                     /* subnormal or zero */
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t half_man = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1u);
    uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (half_man & 1u))) half_man++;
    return (uint16_t)(sign | half_man);
  }
  uint32_t half_man = man >> 13;
  uint32_t rem = man & 0x1fffu;
  uint16_t h = (uint16_t)(sign | ((uint32_t)e << 10) | half_man);
  if (rem > 0x1000u || (rem == 0x1000u && (half_man & 1u))) h++; /* carries into exp */
  return h;
}

float orc_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t x;
  if (exp == 0) {
    if (man == 0) {
      x = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do { man <<= 1; e++; } while (!(man & 0x400u));
      x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 0x1f) {
    x = sign | 0x7f800000u | (man << 13);
  } else {
    x = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

void orc_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = orc_f32_to_f16(src[i]);
}
void orc_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = orc_f16_to_f32(src[i]);
}

/* Correctly rounded f64 -> f16 (ties to even), the single-rounding narrowing
 * of the reference's f16_from_f64 (crates/rocket-npu/src/ops/mod.rs:123-185):
 * scale the magnitude by a power of two so the f16 significand is the integer
 * part, then rint() (ties to even in the default rounding mode). */
uint16_t orc_f64_to_f16(double v) {
  if (isnan(v)) return (uint16_t)(signbit(v) ? 0xfe00u : 0x7e00u);
  const uint16_t sign = signbit(v) ? 0x8000u : 0u;
  const double a = fabs(v);
  if (a >= 65520.0) return (uint16_t)(sign | 0x7c00u); /* rounds past the max finite */
  if (a < 0x1p-14) {                                    /* subnormal range: units of 2^-24 */
    const double q = rint(a * 0x1p24);                  /* may reach 1024 = min normal */
    return (uint16_t)(sign | (uint16_t)q);
  }
  int ex;
  frexp(a, &ex);      /* a = m * 2^ex, m in [0.5, 1) */
  int e = ex - 1;     /* a in [2^e, 2^(e+1)) */
  double sig = rint(ldexp(a, 10 - e)); /* in [1024, 2048] */
  if (sig >= 2048.0) { sig = 1024.0; e += 1; }
  if (e > 15) return (uint16_t)(sign | 0x7c00u);
  return (uint16_t)(sign | (uint16_t)((e + 15) << 10) | (uint16_t)((int)sig - 1024));
}

/* ------------------------------------------------------------------ Q8_0 */
/* Reference encoder: crates/rocket-npu/src/bin/q8_bench.rs:199-219.
 * Per 32-value block along K: d = f16(amax / 127); codes are rounded half
 * away from zero (Rust f32::round) against the stored f16 scale, clamped to
 * [-127, 127]. Writes codes [n, k] and f16 scale bits [n, k/32]. */
void orc_q8_0_quantize(const float* w, int64_t n, int64_t k, int8_t* codes, uint16_t* scales) {
  const int64_t ng = k / 32;
  for (int64_t r = 0; r < n; ++r) {
    for (int64_t g = 0; g < ng; ++g) {
      const float* seg = w + r * k + g * 32;
      float amax = 0.0f;
      for (int i = 0; i < 32; ++i) {
        float a = fabsf(seg[i]);
        amax = (a > amax) ? a : amax; /* Rust f32::max ignores NaN */
      }
      uint16_t d = orc_f32_to_f16(amax / 127.0f);
      float scale = orc_f16_to_f32(d);
      scales[r * ng + g] = d;
      float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
      for (int i = 0; i < 32; ++i) {
        float v = roundf(seg[i] * inv);
        if (v < -127.0f) v = -127.0f;
        if (v > 127.0f) v = 127.0f;
        codes[r * k + g * 32 + i] = (int8_t)v;
      }
    }
  }
}

/* GGUF Q8_0 block layout: src/util/gguf.rs:197-215 — 34 bytes per block,
 * little-endian f16 scale then 32 int8 codes. */
void orc_q8_0_to_blocks(const int8_t* codes, const uint16_t* scales, int64_t n, int64_t k,
                        uint8_t* blocks) {
  const int64_t nb = n * (k / 32);
  for (int64_t b = 0; b < nb; ++b) {
    blocks[b * 34 + 0] = (uint8_t)(scales[b] & 0xffu);
    blocks[b * 34 + 1] = (uint8_t)(scales[b] >> 8);
    memcpy(blocks + b * 34 + 2, codes + b * 32, 32);
  }
}

/* GGUF decode, src/util/gguf.rs:197-215: value = f32(d) * f32(q). */
void orc_q8_0_dequant_blocks(const uint8_t* blocks, int64_t nblocks, float* out) {
  for (int64_t b = 0; b < nblocks; ++b) {
    uint16_t dbits = (uint16_t)(blocks[b * 34] | (blocks[b * 34 + 1] << 8));
    float d = orc_f16_to_f32(dbits);
    for (int i = 0; i < 32; ++i) out[b * 32 + i] = d * (float)(int8_t)blocks[b * 34 + 2 + i];
  }
}

/* Same decode from the planar form (codes [n,k], scales [n,k/32]). */
void orc_q8_0_dequant(const int8_t* codes, const uint16_t* scales, int64_t n, int64_t k,
                      float* out) {
  const int64_t ng = k / 32;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < n; ++r)
    for (int64_t c = 0; c < k; ++c)
      out[r * k + c] = orc_f16_to_f32(scales[r * ng + c / 32]) * (float)codes[r * k + c];
}

/* ------------------------------------------------------------------ GEMMs */
/* Exact-as-possible reference product C[m,n] = sum_k A[m,k] * W[n,k] with f64
 * accumulation (the f64 product the reference's q8_bench gates on,
 * q8_bench.rs:24-31). */
void orc_gemm_f64acc(const float* a, const float* w, int64_t m, int64_t n, int64_t k, float* c) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t j = 0; j < n; ++j) {
      double acc = 0.0;
      const float* ar = a + i * k;
      const float* wr = w + j * k;
      for (int64_t p = 0; p < k; ++p) acc += (double)ar[p] * (double)wr[p];
      c[i * n + j] = (float)acc;
    }
  }
}

/* The `--device cpu` algorithm of the reference's Q8 path: Burn flex's
 * q_matmul dequantises the whole weight and runs an f32 GEMM
 * (docs/experiments/experiment-log.md:109-118; src/commands/gemm.rs:66-83).
 * This is the timed CPU baseline: dequantise, then a cache-blocked f32 GEMM
 * over all OpenMP threads. `wdeq` is caller scratch of n*k floats. */
void orc_q8_0_matmul_cpu(const float* a, const int8_t* codes, const uint16_t* scales, int64_t m,
                         int64_t n, int64_t k, float* wdeq, float* c) {
  orc_q8_0_dequant(codes, scales, n, k, wdeq);
  const int64_t MB = 64, NB = 64;
  const int64_t mt = (m + MB - 1) / MB, nt = (n + NB - 1) / NB;
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int64_t ti = 0; ti < mt; ++ti) {
    for (int64_t tj = 0; tj < nt; ++tj) {
      const int64_t i0 = ti * MB, j0 = tj * NB;
      const int64_t i1 = i0 + MB < m ? i0 + MB : m, j1 = j0 + NB < n ? j0 + NB : n;
      for (int64_t i = i0; i < i1; ++i) {
        const float* ar = a + i * k;
        for (int64_t j = j0; j < j1; ++j) {
          const float* wr = wdeq + j * k;
          float s0 = 0, s1 = 0, s2 = 0, s3 = 0, s4 = 0, s5 = 0, s6 = 0, s7 = 0;
          int64_t p = 0;
          for (; p + 8 <= k; p += 8) {
            s0 += ar[p] * wr[p];
            s1 += ar[p + 1] * wr[p + 1];
            s2 += ar[p + 2] * wr[p + 2];
            s3 += ar[p + 3] * wr[p + 3];
            s4 += ar[p + 4] * wr[p + 4];
            s5 += ar[p + 5] * wr[p + 5];
            s6 += ar[p + 6] * wr[p + 6];
            s7 += ar[p + 7] * wr[p + 7];
          }
          float s = ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7));
          for (; p < k; ++p) s += ar[p] * wr[p];
          c[i * n + j] = s;
        }
      }
    }
  }
}

/* ------------------------------------------------------------------ W8A8 */
/* static_code, ext.rs:1236-1238: clamp(round_ties_even(v * inv), -128, 127). */
static inline int8_t static_code(float v, float inv) {
  float r = rintf(v * inv); /* default rounding mode: ties to even */
  if (r < -128.0f) r = -128.0f;
  if (r > 127.0f) r = 127.0f;
  return (int8_t)r;
}

int8_t orc_static_code(float v, float inv) { return static_code(v, inv); }

/* Per-row activation quantiser of matmul_qat, ext.rs:1263-1279. in_scale == 0:
 * scale = max(amax / 127, 1e-12) per row; else the static in_scale. */
void orc_quantize_rows_i8(const float* x, int64_t m, int64_t k, float in_scale, int8_t* q,
                          float* row_scale) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r) {
    const float* xr = x + r * k;
    float s = in_scale;
    if (in_scale == 0.0f) {
      float amax = 0.0f;
      for (int64_t i = 0; i < k; ++i) {
        float a = fabsf(xr[i]);
        amax = a > amax ? a : amax;
      }
      s = amax / 127.0f;
      if (!(s > 1e-12f)) s = 1e-12f;
    }
    row_scale[r] = s;
    const float inv = 1.0f / s;
    for (int64_t i = 0; i < k; ++i) q[r * k + i] = static_code(xr[i], inv);
  }
}

/* Exact int8 product: acc[m,n] = sum_k q[m,k] * w[n,k] accumulated in int64
 * (the ROCKET_QAT_CHECK recomputation, ext.rs:1309-1334). Returns 0, or -6
 * (RANGE) when an accumulator leaves int32. */
int orc_gemm_i8(const int8_t* q, const int8_t* w, int64_t m, int64_t n, int64_t k, int32_t* acc) {
  int bad = 0;
  if (k <= 131071) {
    /* |q*w| <= 128*128 = 2^14, so any k below 2^17 sums exactly in int32
     * (the same integers as the i64 form below, which checks the range). */
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; ++i) {
      const int8_t* qr = q + i * k;
      for (int64_t j = 0; j < n; ++j) {
        const int8_t* wr = w + j * k;
        int32_t s = 0;
        for (int64_t p = 0; p < k; ++p) s += (int32_t)qr[p] * (int32_t)wr[p];
        acc[i * n + j] = s;
      }
    }
    return 0;
  }
#pragma omp parallel for schedule(static) reduction(| : bad)
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t j = 0; j < n; ++j) {
      int64_t s = 0;
      const int8_t* qr = q + i * k;
      const int8_t* wr = w + j * k;
      for (int64_t p = 0; p < k; ++p) s += (int64_t)qr[p] * (int64_t)wr[p];
      if (s > INT32_MAX || s < INT32_MIN) bad = 1;
      acc[i * n + j] = (int32_t)s;
    }
  }
  return bad ? -6 : 0;
}

/* matmul_qat epilogue, ext.rs:1350-1363: y = f32(acc) * (row_scale * w_scale[n]);
 * with out_scale != 0 the result is rounded to the output int8 grid. */
void orc_w8a8_epilogue(const int32_t* acc, const float* row_scale, const float* w_scale,
                       int64_t m, int64_t n, float out_scale, float* y) {
  const float out_inv = out_scale != 0.0f ? 1.0f / out_scale : 0.0f;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t j = 0; j < n; ++j) {
      float v = (float)acc[i * n + j] * (row_scale[i] * w_scale[j]);
      if (out_scale != 0.0f) v = (float)static_code(v, out_inv) * out_scale;
      y[i * n + j] = v;
    }
  }
}

/* Synthetic per-output-channel weight quantiser used to build W8A8 test
 * weights from float weights: s[n] = max(amax/127, 1e-12), codes
 * clamp(round_ties_even(w / s), -127, 127) (symmetric QAT-style codes). */
void orc_quantize_weight_per_channel(const float* w, int64_t n, int64_t k, int8_t* codes,
                                     float* scale) {
  for (int64_t r = 0; r < n; ++r) {
    float amax = 0.0f;
    for (int64_t i = 0; i < k; ++i) {
      float a = fabsf(w[r * k + i]);
      amax = a > amax ? a : amax;
    }
    float s = amax / 127.0f;
    if (!(s > 1e-12f)) s = 1e-12f;
    scale[r] = s;
    const float inv = 1.0f / s;
    for (int64_t i = 0; i < k; ++i) {
      float v = rintf(w[r * k + i] * inv);
      if (v < -127.0f) v = -127.0f;
      if (v > 127.0f) v = 127.0f;
      codes[r * k + i] = (int8_t)v;
    }
  }
}

/* Group-wise int8 quantiser, crates/burn-rocket/src/host.rs:77-90: per group,
 * scale = max(amax/127, 1e-12), q = clamp(round_half_away(x / scale), ±127). */
void orc_quantize_row_groups(const float* x, int64_t k, int64_t group, int8_t* q, float* s) {
  for (int64_t g = 0; g < k / group; ++g) {
    const float* seg = x + g * group;
    float amax = 0.0f;
    for (int64_t i = 0; i < group; ++i) {
      float a = fabsf(seg[i]);
      amax = a > amax ? a : amax;
    }
    float scale = amax / 127.0f;
    if (!(scale > 1e-12f)) scale = 1e-12f;
    s[g] = scale;
    const float inv = 1.0f / scale;
    for (int64_t i = 0; i < group; ++i) {
      float v = roundf(seg[i] * inv);
      if (v < -127.0f) v = -127.0f;
      if (v > 127.0f) v = 127.0f;
      q[g * group + i] = (int8_t)v;
    }
  }
}

/* ------------------------------------------------------------------ masks */
/* Visibility predicates of crates/burn-rocket/src/masks.rs:11-114 and the
 * MaskMode dispatch of ext.rs:1643-1667, 1768-1804. Mode numbers match
 * RB_MASK_* in include/rocket_b200.h. i, j are chunk-local indices. */
int orc_mask_visible(int mode, int64_t window, int64_t q0, int64_t k0, int64_t i, int64_t j) {
  const int64_t t = q0 + i, key = k0 + j;
  switch (mode) {
    case 0: /* None */
    case 1: /* NoneBlock */
      return 1;
    case 2: /* Causal: j <= t (masks.rs:37-39) */
      return key <= t;
    case 3: /* Window: |t - j| <= w (masks.rs:11-25) */
      if (window < 0) return 1;
      return (t > key ? t - key : key - t) <= window;
    case 4: /* CausalWindow: t - w < j <= t (masks.rs:26-36) */
      if (window < 0) return key <= t;
      return key <= t && t - key < window;
    case 5: /* WindowBlock (masks.rs:92-114) */
      if (window < 0) return 1;
      return (t > key ? t - key : key - t) <= window;
    case 6: /* CausalBlock (masks.rs:58-85) */
      if (window < 0) return key <= t;
      return key <= t && t - key < window;
    default:
      return 0;
  }
}

/* ------------------------------------------------------------------ attention */
/* fa_score, crates/rocket-npu/src/attn/oneshot.rs:193-199. */
static inline float fa_score(float qk, float scale, float softcap, float mask) {
  float s = qk * scale;
  if (softcap != 0.0f) s = softcap * tanhf(s / softcap);
  s = s + mask;
  return s > -30000.0f ? s : -30000.0f;
}

float orc_fa_score(float qk, float scale, float softcap, float mask) {
  return fa_score(qk, scale, softcap, mask);
}

/* flash_attn_ref, crates/rocket-npu/src/attn/oneshot.rs:130-185, restated on
 * the boundary's token-major layout (q/out [n_q, H*D], k/v [n_kv, KV*D], f16
 * bits) instead of the reference's head-major copies (ext.rs:1818-1820, the
 * same values). The QK dot accumulates in f64 and narrows to f32 for
 * fa_score; exp, the row sum and the AV product run in f64; the output is
 * rounded to f16 once. The mask is the predicate of orc_mask_visible (0 or
 * -inf additive). Rows are split across OpenMP threads. */
void orc_flash_attn_ref(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t n_q,
                        int64_t n_kv, int n_head, int n_kv_heads, int head_dim, float scale,
                        float softcap, int mode, int64_t window, int64_t q0, int64_t k0,
                        uint16_t* out) {
  const int gqa = n_head / n_kv_heads;
  const int64_t ldq = (int64_t)n_head * head_dim, ldk = (int64_t)n_kv_heads * head_dim;
  /* f16 -> f64 tables once */
  double* qd = (double*)malloc(sizeof(double) * n_q * ldq);
  double* kd = (double*)malloc(sizeof(double) * n_kv * ldk);
  double* vd = (double*)malloc(sizeof(double) * n_kv * ldk);
  for (int64_t i = 0; i < n_q * ldq; ++i) qd[i] = orc_f16_to_f32(q[i]);
  for (int64_t i = 0; i < n_kv * ldk; ++i) {
    kd[i] = orc_f16_to_f32(k[i]);
    vd[i] = orc_f16_to_f32(v[i]);
  }
#pragma omp parallel
  {
    double* sc = (double*)malloc(sizeof(double) * n_kv);
    double* acc = (double*)malloc(sizeof(double) * head_dim);
#pragma omp for schedule(dynamic, 4) collapse(2)
    for (int h = 0; h < n_head; ++h) {
      for (int64_t t = 0; t < n_q; ++t) {
        const int hk = h / gqa;
        const double* qr = qd + t * ldq + (int64_t)h * head_dim;
        double mx = -INFINITY;
        for (int64_t j = 0; j < n_kv; ++j) {
          const double* kr = kd + j * ldk + (int64_t)hk * head_dim;
          double dot = 0.0;
          for (int d = 0; d < head_dim; ++d) dot += qr[d] * kr[d];
          float m = orc_mask_visible(mode, window, q0, k0, t, j) ? 0.0f : -INFINITY;
          double s = (double)fa_score((float)dot, scale, softcap, m);
          sc[j] = s;
          if (s > mx) mx = s;
        }
        double sum = 0.0;
        for (int64_t j = 0; j < n_kv; ++j) {
          sc[j] = exp(sc[j] - mx);
          sum += sc[j];
        }
        const double inv = sum > 0.0 ? 1.0 / sum : 0.0;
        for (int d = 0; d < head_dim; ++d) acc[d] = 0.0;
        for (int64_t j = 0; j < n_kv; ++j) {
          const double* vr = vd + j * ldk + (int64_t)hk * head_dim;
          const double p = sc[j];
          for (int d = 0; d < head_dim; ++d) acc[d] += p * vr[d];
        }
        uint16_t* o = out + t * ldq + (int64_t)h * head_dim;
        for (int d = 0; d < head_dim; ++d) {
          const uint16_t hbits = orc_f64_to_f16(acc[d] * inv);
          o[d] = hbits;
        }
      }
    }
    free(sc);
    free(acc);
  }
  free(qd);
  free(kd);
  free(vd);
}

/* Tiled f32 online-softmax attention over all OpenMP threads: the timed CPU
 * baseline for the attention op (the algorithm of the reference's fused CPU
 * path and of its tiled NPU fold, attn/mod.rs:78-101, 926-1004), f32
 * throughout, causal tile skipping. Same layout and semantics as above. */
void orc_attention_cpu(const float* q, const float* k, const float* v, int64_t n_q, int64_t n_kv,
                       int n_head, int n_kv_heads, int head_dim, float scale, int causal,
                       float* out) {
  const int gqa = n_head / n_kv_heads;
  const int64_t ldq = (int64_t)n_head * head_dim, ldk = (int64_t)n_kv_heads * head_dim;
  const int64_t QB = 32;
#pragma omp parallel
  {
    float* s = (float*)malloc(sizeof(float) * QB * 64);
    float* o = (float*)malloc(sizeof(float) * QB * head_dim);
    float* m = (float*)malloc(sizeof(float) * QB);
    float* l = (float*)malloc(sizeof(float) * QB);
#pragma omp for schedule(dynamic) collapse(2)
    for (int h = 0; h < n_head; ++h) {
      for (int64_t t0 = 0; t0 < n_q; t0 += QB) {
        const int hk = h / gqa;
        const int64_t tq = (n_q - t0) < QB ? (n_q - t0) : QB;
        for (int64_t i = 0; i < tq; ++i) {
          m[i] = -INFINITY;
          l[i] = 0.0f;
          for (int d = 0; d < head_dim; ++d) o[i * head_dim + d] = 0.0f;
        }
        const int64_t jend = causal ? (t0 + tq < n_kv ? t0 + tq : n_kv) : n_kv;
        for (int64_t j0 = 0; j0 < jend; j0 += 64) {
          const int64_t tk = (jend - j0) < 64 ? (jend - j0) : 64;
          for (int64_t i = 0; i < tq; ++i) {
            const float* qr = q + (t0 + i) * ldq + (int64_t)h * head_dim;
            float mx = m[i];
            for (int64_t j = 0; j < tk; ++j) {
              const float* kr = k + (j0 + j) * ldk + (int64_t)hk * head_dim;
              float dot = 0.0f;
              for (int d = 0; d < head_dim; ++d) dot += qr[d] * kr[d];
              float sv = dot * scale;
              if (causal && j0 + j > t0 + i) sv = -30000.0f;
              if (sv < -30000.0f) sv = -30000.0f;
              s[i * 64 + j] = sv;
              if (sv > mx) mx = sv;
            }
            const float alpha = expf(m[i] - mx);
            float* orow = o + i * head_dim;
            for (int d = 0; d < head_dim; ++d) orow[d] *= alpha;
            float sum = l[i] * alpha;
            for (int64_t j = 0; j < tk; ++j) {
              const float p = expf(s[i * 64 + j] - mx);
              sum += p;
              const float* vr = v + (j0 + j) * ldk + (int64_t)hk * head_dim;
              for (int d = 0; d < head_dim; ++d) orow[d] += p * vr[d];
            }
            l[i] = sum;
            m[i] = mx;
          }
        }
        for (int64_t i = 0; i < tq; ++i) {
          float* dst = out + (t0 + i) * ldq + (int64_t)h * head_dim;
          const float inv = 1.0f / l[i];
          for (int d = 0; d < head_dim; ++d) dst[d] = o[i * head_dim + d] * inv;
        }
      }
    }
    free(s);
    free(o);
    free(m);
    free(l);
  }
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Thread count of the later parallel regions (a launcher such as torchrun sets
 * OMP_NUM_THREADS=1 in every rank; the CPU baseline wants all host cores). */
void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
