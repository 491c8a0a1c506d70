/* CPU oracle for the diffucore_b200 hot path. TEST INFRASTRUCTURE ONLY: the tests,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm call it as the checker or
 * as the timed CPU restatement; the product path never loads it.
 *
 * Each function restates the reference's arithmetic (diffucore 0.2.4) at the cited lines:
 *   - per-row int8 quantizer: src/diffucore/models/_int8.py:87-97 (`_quantize_rows`), the torch-op
 *     path that runs on CPU; IEEE fp32 division, round-half-even, clamp.
 *   - ConvRot rotation: _int8.py:364-372 (`_hadamard_rows`), radix-4 stages most significant
 *     digit first, y = S - 2 x[3 - d], S = (x0 + x1) + (x2 + x3), then * 0.0625. The summation
 *     order of S is the one the CUDA kernel defines (the Triton source leaves it open).
 *   - int32 GEMM: torch._int_mm (_int8.py:200-207), exact.
 *   - rescale: _int8.py:313-323: y = dtype(float(acc) * (sx * sw)); y = dtype(float(y) + bias).
 *   - attention prep: src/diffucore/kernels/int8_attn_sm80.cu:92-142 (K column sums, fixed
 *     order), :38-90 (K codes, mean subtracted as one fused multiply-add), :341-388 (Q codes).
 *   - attention: softmax(S * sq * sk * sm_scale) V in double over the exact int32 S, i.e. the
 *     ideal result of the reference's quantization.
 * Build: gcc -O2 -fopenmp -ffp-contract=off -shared -fPIC (contraction off so every a*b+c below
 * rounds twice unless written as fmaf).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_F32 0
#define OR_F16 1
#define OR_BF16 2

/* ------------------------------------------------------------------ 16-bit floats */

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);                                          /* round half to even */
  return (uint16_t)(u >> 16);
}

static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else { /* subnormal: normalise */
      exp = 127 - 15 + 1;
      while ((man & 0x400u) == 0) { man <<= 1; exp--; }
      man &= 0x3ffu;
      u = sign | (exp << 23) | (man << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7f800000u | (man << 13);
  } else {
    u = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t f32_to_f16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  const uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);   /* rounds to >= 65520: inf */
  if (a < 0x38800000u) {                                     /* below 2^-14: subnormal half */
    if (a < 0x33000000u) return sign;                        /* below 2^-25: rounds to 0 */
    const int e = (int)(a >> 23);
    const uint32_t m = (a & 0x7fffffu) | 0x800000u;
    /* value = m * 2^(e - 150); the half subnormal unit is 2^-24, so q = m * 2^(e - 126) */
    const int rs = 126 - e;                                  /* right shift, 14..24 */
    uint32_t q = m >> rs;
    const uint32_t rem = m & ((1u << rs) - 1u), half = 1u << (rs - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t q = ((a >> 13) - ((127 - 15) << 10));
  const uint32_t rem = a & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

static float load_elem(const void* base, int dtype, int64_t idx) {
  if (dtype == OR_BF16) return bf16_to_f32(((const uint16_t*)base)[idx]);
  if (dtype == OR_F16) return f16_to_f32(((const uint16_t*)base)[idx]);
  return ((const float*)base)[idx];
}

static float round_dtype(float x, int dtype) {
  if (dtype == OR_BF16) return bf16_to_f32(f32_to_bf16(x));
  if (dtype == OR_F16) return f16_to_f32(f32_to_f16(x));
  return x;
}

void or_round_to(const float* x, int64_t n, int dtype, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = dtype == OR_BF16 ? f32_to_bf16(x[i]) : f32_to_f16(x[i]);
}

void or_to_float(const uint16_t* x, int64_t n, int dtype, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = load_elem(x, dtype, i);
}

/* ------------------------------------------------------------------ quantizer */

static float gelu_dtype(float h, int mode, int dtype) {
  if (mode == 1) {
    const float t = h * 0.7071067811865476f;
    const float e = 1.0f + erff(t);
    return round_dtype((0.5f * h) * e, dtype);
  }
  if (mode == 2) {
    const float h3 = (h * h) * h;
    const float inner = 0.7978845608028654f * (h + 0.044715f * h3);
    const float e = 1.0f + tanhf(inner);
    return round_dtype((0.5f * h) * e, dtype);
  }
  return h;
}

/* The four-term sums of each stage follow the order the reference's Triton `_hadamard_rows`
 * uses, which its register layout decides from the kernel's block width BLOCK = the next power
 * of two >= the row width (inferred on a B200 from `_rot_quant_kernel`'s own scales):
 *   BLOCK 256:     d3, d2, d1 (x0 + x2) + (x1 + x3); d0 (x0 + x1) + (x2 + x3)
 *   BLOCK 512:     d3 (x0 + x1) + (x2 + x3); d2, d1 (x0 + x2) + (x1 + x3); d0 ((x0 + x1) + x2) + x3
 *   BLOCK 1024:    d3, d2 (x0 + x2) + (x1 + x3); d1 (x0 + x1) + (x2 + x3); d0 in sequence
 *   BLOCK >= 2048: d3, d2 (x0 + x2) + (x1 + x3); d1, d0 in sequence */
enum { SUM_P0123 = 0, SUM_P0213 = 1, SUM_S0123 = 2 };

static int stage_order(int64_t width, int stage) {
  int64_t block = 256;
  while (block < width) block <<= 1;
  static const int table[4][4] = {   /* [block class][stage d0..d3] */
      {SUM_P0123, SUM_P0213, SUM_P0213, SUM_P0213},
      {SUM_S0123, SUM_P0213, SUM_P0213, SUM_P0123},
      {SUM_S0123, SUM_P0123, SUM_P0213, SUM_P0213},
      {SUM_S0123, SUM_S0123, SUM_P0213, SUM_P0213}};
  const int cls = block <= 256 ? 0 : block == 512 ? 1 : block == 1024 ? 2 : 3;
  return table[cls][stage];
}

/* One 256-wide group in place, of a row `width` elements wide; digit d of index e (base 4, d3
 * most significant) has stride 4^d. Stages d3, d2, d1, d0 (_int8.py:364-372: reshape to
 * [., 4, 4, 4, 4], then per axis sum - 2 * flip, then x 0.0625). */
void or_hadamard256(float* x, int64_t width) {
  float y[256];
  for (int stage = 3; stage >= 0; --stage) {
    const int stride = 1 << (2 * stage);
    const int ord = stage_order(width, stage);
    for (int e = 0; e < 256; ++e) {
      const int d = (e / stride) & 3;
      const int base = e - d * stride;
      const float x0 = x[base], x1 = x[base + stride], x2 = x[base + 2 * stride], x3 = x[base + 3 * stride];
      float s;
      if (ord == SUM_P0213) s = (x0 + x2) + (x1 + x3);
      else if (ord == SUM_S0123) s = ((x0 + x1) + x2) + x3;
      else s = (x0 + x1) + (x2 + x3);
      y[e] = s - 2.0f * x[base + (3 - d) * stride];
    }
    memcpy(x, y, sizeof(y));
  }
  for (int e = 0; e < 256; ++e) x[e] = x[e] * 0.0625f;
}

static int8_t quant_code(float x, float scale) {
  float t = rintf(x / scale);
  if (t < -128.0f) t = -128.0f;
  if (t > 127.0f) t = 127.0f;
  return (int8_t)(int)t;
}

/* x [M, K] (row stride ldx, dtype) -> q [M, K], s [M]. group 0 or 256; gelu 0/1/2. */
void or_quant_rows(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx, int group, int gelu,
                   int8_t* q, float* s) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    float* row = (float*)malloc(sizeof(float) * (size_t)K);
    for (int64_t k = 0; k < K; ++k) row[k] = gelu_dtype(load_elem(x, dtype, m * ldx + k), gelu, dtype);
    if (group == 256)
      for (int64_t g = 0; g + 256 <= K; g += 256) or_hadamard256(row + g, K);
    float amax = 0.0f;
    for (int64_t k = 0; k < K; ++k) amax = fmaxf(amax, fabsf(row[k]));
    float scale = amax / 127.0f;
    if (scale < 1e-30f) scale = 1e-30f;
    for (int64_t k = 0; k < K; ++k) q[m * K + k] = quant_code(row[k], scale);
    s[m] = scale;
    free(row);
  }
}

/* ------------------------------------------------------------------ GEMM */

void or_int_mm(const int8_t* q, const int8_t* w, int64_t M, int64_t N, int64_t K, int32_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    const int8_t* a = q + m * K;
    for (int64_t n = 0; n < N; ++n) {
      const int8_t* b = w + n * K;
      int32_t acc = 0;
      for (int64_t k = 0; k < K; ++k) acc += (int32_t)a[k] * (int32_t)b[k];
      out[m * N + n] = acc;
    }
  }
}

/* bias: 16-bit bits in out dtype, or NULL. out: 16-bit bits. gelu 0/1/2 applied after bias. */
void or_rescale(const int32_t* acc, const float* sx, const float* sw, const uint16_t* bias, int dtype, int64_t M,
                int64_t N, int gelu, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      const float a = (float)acc[m * N + n];
      const float sc = sx[m] * sw[n];
      float y = round_dtype(a * sc, dtype);
      if (bias != NULL) y = round_dtype(y + load_elem(bias, dtype, n), dtype);
      y = gelu_dtype(y, gelu, dtype);
      out[m * N + n] = dtype == OR_BF16 ? f32_to_bf16(y) : f32_to_f16(y);
    }
  }
}

/* ------------------------------------------------------------------ attention */

/* Element (b, l, h, d) of a (B, L, H, D) tensor with element strides s[3] (stride_d = 1). */
static float at(const void* t, int dtype, const int64_t* s, int64_t b, int64_t l, int64_t h, int64_t d) {
  return load_elem(t, dtype, b * s[0] + l * s[1] + h * s[2] + d);
}

/* K column sums in the reference's fixed order: windows of 128 rows; inside a window 16 row
 * groups rg each add rows r0+rg, r0+rg+16, ...; the 16 partials add in order; windows add in
 * order. ksum [B*H, D]. */
void or_attn_ksum(const void* k, int dtype, int64_t B, int64_t H, int64_t L, int64_t D, const int64_t* ks,
                  float* ksum) {
  const int64_t nwin = (L + 127) / 128;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t b = 0; b < B; ++b)
    for (int64_t h = 0; h < H; ++h)
      for (int64_t d = 0; d < D; ++d) {
        float total = 0.0f;
        for (int64_t w = 0; w < nwin; ++w) {
          const int64_t r0 = w * 128, r1 = r0 + 128 < L ? r0 + 128 : L;
          float win = 0.0f;
          for (int rg = 0; rg < 16; ++rg) {
            float part = 0.0f;
            for (int64_t r = r0 + rg; r < r1; r += 16) part += at(k, dtype, ks, b, r, h, d);
            win += part;
          }
          total += win;
        }
        ksum[(b * H + h) * D + d] = total;
      }
}

/* Per-64-row block codes of x (B, L, H, D): x' = fma(-ksum, 1/L, x) when ksum != NULL;
 * amax over the block; scale = amax / 127; code = rint(x' * (127 / amax)) (0 if amax == 0).
 * codes [B*H, L, D], scales [B*H, ceil(L / 64)]. */
void or_attn_block_quant(const void* x, int dtype, int64_t B, int64_t H, int64_t L, int64_t D, const int64_t* xs,
                         const float* ksum, int8_t* codes, float* scales) {
  const int64_t nblk = (L + 63) / 64;
  const float inv_l = 1.0f / (float)L;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t bh = 0; bh < B * H; ++bh)
    for (int64_t blk = 0; blk < nblk; ++blk) {
      const int64_t b = bh / H, h = bh % H;
      const int64_t r0 = blk * 64, r1 = r0 + 64 < L ? r0 + 64 : L;
      float amax = 0.0f;
      for (int64_t r = r0; r < r1; ++r)
        for (int64_t d = 0; d < D; ++d) {
          float v = at(x, dtype, xs, b, r, h, d);
          if (ksum != NULL) v = fmaf(-ksum[bh * D + d], inv_l, v);
          amax = fmaxf(amax, fabsf(v));
        }
      const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
      scales[bh * nblk + blk] = amax / 127.0f;
      for (int64_t r = r0; r < r1; ++r)
        for (int64_t d = 0; d < D; ++d) {
          float v = at(x, dtype, xs, b, r, h, d);
          if (ksum != NULL) v = fmaf(-ksum[bh * D + d], inv_l, v);
          codes[(bh * L + r) * D + d] = (int8_t)(int)rintf(v * inv);
        }
    }
}

/* Per-token codes: amax over D; inv = 127 / amax (0 if amax == 0); code = rint(x * inv);
 * scale = amax / 127. codes [B*H, L, D], scales [B*H, L]. */
void or_attn_token_quant(const void* x, int dtype, int64_t B, int64_t H, int64_t L, int64_t D, const int64_t* xs,
                         int8_t* codes, float* scales) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t bh = 0; bh < B * H; ++bh)
    for (int64_t r = 0; r < L; ++r) {
      const int64_t b = bh / H, h = bh % H;
      float amax = 0.0f;
      for (int64_t d = 0; d < D; ++d) amax = fmaxf(amax, fabsf(at(x, dtype, xs, b, r, h, d)));
      const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
      for (int64_t d = 0; d < D; ++d)
        codes[(bh * L + r) * D + d] = (int8_t)(int)rintf(at(x, dtype, xs, b, r, h, d) * inv);
      scales[bh * L + r] = amax / 127.0f;
    }
}

/* Attention from codes: out[b, i, h, :] = sum_j softmax_j(S_ij * qscale_i * kscale_j * sm_scale) v_j
 * with exact int32 S and double softmax / P.V. qscale per row [B*H, Lq]; kscale per 64-key block
 * [B*H, ceil(Lk/64)]. v (B, Lk, H, D) in dtype with strides vs. out fp32 (B, Lq, H, D) contiguous. */
void or_attn_from_codes(const int8_t* qc, const float* qscale, const int8_t* kc, const float* kscale, const void* v,
                        int dtype, const int64_t* vs, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D,
                        double sm_scale, float* out) {
  const int64_t nkb = (Lk + 63) / 64;
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
  for (int64_t bh = 0; bh < B * H; ++bh)
    for (int64_t i = 0; i < Lq; ++i) {
      const int64_t b = bh / H, h = bh % H;
      double* logit = (double*)malloc(sizeof(double) * (size_t)Lk);
      double* acc = (double*)calloc((size_t)D, sizeof(double));
      const int8_t* qi = qc + (bh * Lq + i) * D;
      double mx = -INFINITY;
      for (int64_t j = 0; j < Lk; ++j) {
        const int8_t* kj = kc + (bh * Lk + j) * D;
        int32_t s = 0;
        for (int64_t d = 0; d < D; ++d) s += (int32_t)qi[d] * (int32_t)kj[d];
        logit[j] = (double)s * (double)qscale[bh * Lq + i] * (double)kscale[bh * nkb + j / 64] * sm_scale;
        if (logit[j] > mx) mx = logit[j];
      }
      double denom = 0.0;
      for (int64_t j = 0; j < Lk; ++j) {
        const double p = exp(logit[j] - mx);
        denom += p;
        for (int64_t d = 0; d < D; ++d) acc[d] += p * (double)at(v, dtype, vs, b, j, h, d);
      }
      for (int64_t d = 0; d < D; ++d) out[((b * Lq + i) * H + h) * D + d] = (float)(acc[d] / denom);
      free(logit);
      free(acc);
    }
}

/* Exact fp64 attention (no quantization) for reference-style error checks. */
void or_attn_exact(const void* q, const void* k, const void* v, int dtype, const int64_t* qs, const int64_t* ks,
                   const int64_t* vs, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D, double sm_scale,
                   float* out) {
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
  for (int64_t bh = 0; bh < B * H; ++bh)
    for (int64_t i = 0; i < Lq; ++i) {
      const int64_t b = bh / H, h = bh % H;
      double* logit = (double*)malloc(sizeof(double) * (size_t)Lk);
      double* acc = (double*)calloc((size_t)D, sizeof(double));
      double mx = -INFINITY;
      for (int64_t j = 0; j < Lk; ++j) {
        double s = 0.0;
        for (int64_t d = 0; d < D; ++d) s += (double)at(q, dtype, qs, b, i, h, d) * (double)at(k, dtype, ks, b, j, h, d);
        logit[j] = s * sm_scale;
        if (logit[j] > mx) mx = logit[j];
      }
      double denom = 0.0;
      for (int64_t j = 0; j < Lk; ++j) {
        const double p = exp(logit[j] - mx);
        denom += p;
        for (int64_t d = 0; d < D; ++d) acc[d] += p * (double)at(v, dtype, vs, b, j, h, d);
      }
      for (int64_t d = 0; d < D; ++d) out[((b * Lq + i) * H + h) * D + d] = (float)(acc[d] / denom);
      free(logit);
      free(acc);
    }
}
