// Per-row symmetric int8 quantizer with optional 256-wide ConvRot (Hadamard) rotation and
// optional GELU applied first. HBM-bound: one read of the row, one int8 write, one scale.
//
// Arithmetic follows the reference's torch-op path bit for bit
// (src/diffucore/models/_int8.py:87-97 `_quantize_rows`, :393-397 `_store_quantized`):
//   scale = max(amax / 127, 1e-30)     (IEEE fp32 division)
//   q     = clamp(rint(x / scale), -128, 127)   (IEEE division, round half to even)
// The rotation is the radix-4 butterfly of `_hadamard_rows` (_int8.py:364-372): for each base-4
// digit of the in-group index, most significant first, y = S - 2 * x[digit -> 3 - digit] with
// S = (x[d=0] + x[d=1]) + (x[d=2] + x[d=3]); then y * 0.0625. That summation order is this
// library's definition; the CPU oracle restates it.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "sm100.cuh"

namespace dc {

enum GeluMode : int { kGeluNone = 0, kGeluErf = 1, kGeluTanh = 2 };

template <typename T> struct Vec8;
template <> struct Vec8<__nv_bfloat16> {
  __device__ static void load(const __nv_bfloat16* p, float (&f)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) { float2 t = __bfloat1622float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
  }
  __device__ static void from_raw(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) { f[2 * i] = __uint_as_float(w[i] << 16); f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u); }
  }
  __device__ static float half_bits_to_float(uint32_t h) { return __uint_as_float(h << 16); }
  __device__ static float one(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  __device__ static float round_trip(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};
template <> struct Vec8<__half> {
  __device__ static void load(const __half* p, float (&f)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) { float2 t = __half22float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
  }
  __device__ static void from_raw(const uint4& u, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) { float2 t = __half22float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
  }
  __device__ static float half_bits_to_float(uint32_t h) { return __half2float(__ushort_as_half(static_cast<unsigned short>(h))); }
  __device__ static float one(const __half* p) { return __half2float(*p); }
  __device__ static float round_trip(float x) { return __half2float(__float2half_rn(x)); }
};
template <> struct Vec8<float> {
  __device__ static void load(const float* p, float (&f)[8]) {
    float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  __device__ static void from_raw(const uint4& u, float (&f)[8]) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y); f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
    f[4] = f[5] = f[6] = f[7] = 0.0f;   // unused: raw fp32 rows are not kept
  }
  __device__ static float half_bits_to_float(uint32_t h) { return __uint_as_float(h); }
  __device__ static float one(const float* p) { return *p; }
  __device__ static float round_trip(float x) { return x; }
};

// GELU of a value already in the model dtype, rounded back to that dtype (the reference's
// `_gelu`, _int8.py:432-434, and FLUX's tanh form, nn.GELU(approximate="tanh")).
template <typename T>
__device__ __forceinline__ float gelu_dtype(float h, int mode) {
  if (mode == kGeluErf) {
    const float t = __fmul_rn(h, 0.7071067811865476f);
    const float e = __fadd_rn(1.0f, erff(t));
    return Vec8<T>::round_trip(__fmul_rn(__fmul_rn(0.5f, h), e));
  }
  if (mode == kGeluTanh) {
    // 0.5 * h * (1 + tanh(u)), u = sqrt(2/pi) * (h + 0.044715 * h^3), computed through the
    // identity 0.5 * (1 + tanh(u)) = 1 / (1 + e^(-2u)): h / (1 + 2^(-2 u log2 e)) with one MUFU
    // exp2 and one MUFU reciprocal (relative error ~1e-6, no cancellation for negative h), then
    // rounded to the 16-bit dtype like torch's GELU.
    const float h3 = __fmul_rn(__fmul_rn(h, h), h);
    const float u = __fmul_rn(0.7978845608028654f, __fadd_rn(h, __fmul_rn(0.044715f, h3)));
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(-2.8853900817779268f, u)));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.0f, e)));
    return Vec8<T>::round_trip(__fmul_rn(h, r));
  }
  return h;
}

// The four-term sums of the 256-wide ConvRot butterfly. The reference's Triton `_hadamard_rows`
// (src/diffucore/models/_int8.py:364-372) sums each radix-4 stage (digit d3 of stride 64, d2 of 16,
// d1 of 4, d0 of 1) in an order its register layout decides, and that layout depends on the
// kernel's block width BLOCK = the next power of two >= K (with 4 warps up to BLOCK 2048, 8 above:
// elements a thread holds in a row are summed in sequence, elements in other lanes by butterfly
// shuffles, high lane bit first). Inferred on a B200 from `_rot_quant_kernel`'s own scales over
// 34816-262144 rows per width (the only order per width that matches every row):
//   BLOCK 256:      d3 (x0 + x2) + (x1 + x3), d2 and d1 the same, d0 (x0 + x1) + (x2 + x3)
//   BLOCK 512:      d3 (x0 + x1) + (x2 + x3), d2 and d1 (x0 + x2) + (x1 + x3), d0 ((x0 + x1) + x2) + x3
//   BLOCK 1024:     d3 and d2 (x0 + x2) + (x1 + x3), d1 (x0 + x1) + (x2 + x3), d0 in sequence
//   BLOCK >= 2048:  d3 and d2 (x0 + x2) + (x1 + x3), d1 and d0 in sequence
// An order is packed two bits per stage (stage s = digit d_s at bits 2 s).
constexpr int kSumP0123 = 0;       // (x0 + x1) + (x2 + x3)
constexpr int kSumP0213 = 1;       // (x0 + x2) + (x1 + x3)
constexpr int kSumS0123 = 2;       // ((x0 + x1) + x2) + x3

__host__ __device__ constexpr int rot_pack(int d3, int d2, int d1, int d0) {
  return d0 | (d1 << 2) | (d2 << 4) | (d3 << 6);
}
__host__ __device__ constexpr int rot_stage(int packed, int stage) { return (packed >> (2 * stage)) & 3; }

constexpr int kRotOrder256 = rot_pack(kSumP0213, kSumP0213, kSumP0213, kSumP0123);
constexpr int kRotOrder512 = rot_pack(kSumP0123, kSumP0213, kSumP0213, kSumS0123);
constexpr int kRotOrder1024 = rot_pack(kSumP0213, kSumP0213, kSumP0123, kSumS0123);
constexpr int kRotOrderWide = rot_pack(kSumP0213, kSumP0213, kSumS0123, kSumS0123);   // BLOCK >= 2048

__host__ __device__ inline int rot_order_for_width(int64_t K) {
  int64_t block = 256;
  while (block < K) block <<= 1;
  if (block <= 256) return kRotOrder256;
  if (block == 512) return kRotOrder512;
  if (block == 1024) return kRotOrder1024;
  return kRotOrderWide;
}

// s - 2 x with one rounding. 2 x is exact, so this equals the reference's `sum - 2 * flip`
// computed as a product and a difference (no contraction) bit for bit, in one instruction.
__device__ __forceinline__ float sub_twice(float s, float x) { return __fmaf_rn(-2.0f, x, s); }

__device__ __forceinline__ float quad_sum_ord(float a0, float a1, float a2, float a3, int ord) {
  if (ord == kSumP0213) return __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
  if (ord == kSumS0123) return __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
  return __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
}
__device__ __forceinline__ float2 quad_sum_ord2(float2 a0, float2 a1, float2 a2, float2 a3, int ord) {
  if (ord == kSumP0213) return __fadd2_rn(__fadd2_rn(a0, a2), __fadd2_rn(a1, a3));
  if (ord == kSumS0123) return __fadd2_rn(__fadd2_rn(__fadd2_rn(a0, a1), a2), a3);
  return __fadd2_rn(__fadd2_rn(a0, a1), __fadd2_rn(a2, a3));
}

// One radix-4 stage across lanes: the digit lives in lane bits (xor masks m_lo, m_hi for its low
// and high bit). The first shuffle pairs the lanes whose digits differ in the bit `first` selects,
// the second adds the pair sums: first = m_lo gives (x0 + x1) + (x2 + x3), first = m_hi gives
// (x0 + x2) + (x1 + x3). m_lo | m_hi selects the lane holding digit 3 - d.
__device__ __forceinline__ float hstage_lanes(float x, int m_lo, int m_hi, int first) {
  const int second = first == m_lo ? m_hi : m_lo;
  const float a = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, first));
  const float s = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, second));
  const float f = __shfl_xor_sync(0xffffffffu, x, m_lo | m_hi);          // x[3 - d]
  return sub_twice(s, f);
}

// Rotate the 8 values a lane holds; 32 lanes of a warp hold one 256-wide group, element
// e = lane * 8 + j. Digits: d0 = j & 3, d1 = ((lane & 1) << 1) | (j >> 2), d2 = (lane >> 1) & 3,
// d3 = lane >> 3. Stage order d3, d2, d1, d0 (most significant first); `order` from
// rot_order_for_width (its d3 and d2 sums are always one of the two pair forms).
__device__ __forceinline__ void hadamard256_warp(float (&x)[8], int order) {
  const int o3 = rot_stage(order, 3), o2 = rot_stage(order, 2), o1 = rot_stage(order, 1), o0 = rot_stage(order, 0);
  // d3: lane bits 3 and 4.
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] = hstage_lanes(x[j], 8, 16, o3 == kSumP0123 ? 8 : 16);
  // d2: lane bits 1 and 2.
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] = hstage_lanes(x[j], 2, 4, o2 == kSumP0123 ? 2 : 4);
  // d1: low bit is j bit 2 (in-thread), high bit is lane bit 0; x0, x1 in the even lane of a pair.
  {
    const bool odd = (threadIdx.x & 1) != 0;
    float y[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = x[j], hi = x[j + 4];
      const float plo = __shfl_xor_sync(0xffffffffu, lo, 1), phi = __shfl_xor_sync(0xffffffffu, hi, 1);
      const float x0 = odd ? plo : lo, x1 = odd ? phi : hi, x2 = odd ? lo : plo, x3 = odd ? hi : phi;
      const float s = quad_sum_ord(x0, x1, x2, x3, o1);
      // this lane holds digits 2 odd (j) and 2 odd + 1 (j + 4): x[3 - d] is x3 / x2, or x1 / x0
      y[j] = sub_twice(s, odd ? x1 : x3);
      y[j + 4] = sub_twice(s, odd ? x0 : x2);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = y[j];
  }
  // d0: j bits 0 and 1, all in-thread.
  {
    float y[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float s = quad_sum_ord(x[4 * h], x[4 * h + 1], x[4 * h + 2], x[4 * h + 3], o0);
#pragma unroll
      for (int d = 0; d < 4; ++d) y[4 * h + d] = sub_twice(s, x[4 * h + (3 - d)]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = __fmul_rn(y[j], 0.0625f);
  }
}

// Where element c of row r lives. Plain rows (SEG false): x + r * ldx + c. Segmented rows: the
// first k1 elements are spread over segments of seg_len elements, segment i starting at
// x + i * seg_stride (row r at + r * ldx inside it); elements k1.. come from x2 + r * ldx2 + (c - k1).
// The segmented form reads an all-to-all's receive buffer [P, rows, seg_len] (and a second operand
// concatenated after it) as one row without a copy. seg_len and k1 are multiples of 8.
struct RowSrc {
  const void* x;
  int64_t ldx;
  int seg_len;
  int64_t seg_stride;
  int k1;
  const void* x2;
  int64_t ldx2;
  int full_div;       // 1: the quantizer divides with div.full.f32 (see row_scale)
  int rot_order;      // ConvRot summation order for the row width (rot_order_for_width)
};

__host__ __device__ inline RowSrc plain_rows(const void* x, int64_t ldx) {
  RowSrc r;
  r.x = x; r.ldx = ldx; r.seg_len = 0; r.seg_stride = 0; r.k1 = 0; r.x2 = nullptr; r.ldx2 = 0; r.full_div = 0;
  r.rot_order = 0;
  return r;
}

template <typename T, bool SEG>
__device__ __forceinline__ const T* src_ptr(const RowSrc& s, int64_t row, int c) {
  if (!SEG) return static_cast<const T*>(s.x) + row * s.ldx + c;
  if (c < s.k1) {
    const int seg = c / s.seg_len;
    return static_cast<const T*>(s.x) + seg * s.seg_stride + row * s.ldx + (c - seg * s.seg_len);
  }
  return static_cast<const T*>(s.x2) + row * s.ldx2 + (c - s.k1);
}

// The two divisions of the per-row quantizer, scale = max(amax / 127, 1e-30) and
// code = clamp(rint(x / scale), -128, 127), in one of two arithmetics:
//   IEEE (full = 0): correctly rounded quotients, the reference's torch-op path as it runs on the
//     CPU (src/diffucore/models/_int8.py:87-97), which the CPU oracle restates and the golden
//     vectors pin;
//   FULL (full = 1): the PTX full-range approximate division (div.full.f32) for both quotients, the
//     arithmetic of the reference's Triton quantizers (`_store_quantized`, _int8.py:393-397), which
//     is what the reference runs on a GPU; measured on a B200 to give their codes and scales bit
//     for bit (the reference's GPU torch-op path, amax * (1/127) and IEEE codes, differs from both).
__device__ __forceinline__ float div_full(float a, float b) {
  float r;
  asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ float row_scale(float amax, int full) {
  return fmaxf(full ? div_full(amax, 127.0f) : __fdiv_rn(amax, 127.0f), 1e-30f);
}

__device__ __forceinline__ int8_t quant_code(float x, float scale, int full = 0) {
  float t = rintf(full ? div_full(x, scale) : __fdiv_rn(x, scale));
  t = fminf(fmaxf(t, -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(t));
}

// Eight codes without a division or a float->int conversion on the common path. y = x * (1 / scale)
// is within ~2^-23 relative (|y| <= 127.5, so within 2e-5 absolute) of the IEEE quotient x / scale;
// t = y + 1.5 * 2^23 rounds y to an integer with ties to even (the float grid there has unit
// spacing), and the code is the low byte of t's bits (|codes| <= 127, so no clamp is reached).
// When some y lies within 1e-4 of a rounding boundary k + 1/2, the quotient and y might round
// differently, so those eight values are redone with the exact division (quant_code). The result
// is bit-identical to quant_code on every element.
constexpr float kRoundMagic = 12582912.0f;      // 1.5 * 2^23

// Low byte of rn(y) for |y| <= 127.5 (a code): y + 1.5 * 2^23 rounds y to an integer with ties to
// even, exactly as __float2int_rn, on the FMA pipe instead of the conversion unit.
__device__ __forceinline__ uint32_t code_byte(float y) {
  return __float_as_uint(__fadd_rn(y, kRoundMagic)) & 0xFFu;
}

__device__ __forceinline__ uint2 quant8(const float (&v)[8], float scale, float inv_scale, int full = 0) {
  uint32_t b[8];
  if (full) {
#pragma unroll
    for (int j = 0; j < 8; ++j) b[j] = static_cast<uint32_t>(static_cast<uint8_t>(quant_code(v[j], scale, 1)));
    return make_uint2(__byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410),
                      __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410));
  }
  uint32_t d[8];     // |y - rint(y)| as sign-cleared float bits: unsigned order == magnitude order
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float y = __fmul_rn(v[j], inv_scale);
    const float t = __fadd_rn(y, kRoundMagic);
    d[j] = __float_as_uint(__fsub_rn(y, __fsub_rn(t, kRoundMagic))) & 0x7FFFFFFFu;
    b[j] = __float_as_uint(t);
  }
  const uint32_t dmax = max(max(max(d[0], d[1]), max(d[2], d[3])), max(max(d[4], d[5]), max(d[6], d[7])));
  if (dmax > __float_as_uint(0.5f - 1e-4f)) {
#pragma unroll
    for (int j = 0; j < 8; ++j) b[j] = static_cast<uint32_t>(static_cast<uint8_t>(quant_code(v[j], scale)));
  }
  // low bytes of b[0..3] -> w0, b[4..7] -> w1
  const uint32_t w0 = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
  const uint32_t w1 = __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410);
  return make_uint2(w0, w1);
}

// Warp-per-row quantizer for K <= 32 * 8 * VPT (K % 8 == 0, 16-byte aligned rows): the amax
// reduction is warp shuffles only and a CTA holds several rows at once. Without rotation or GELU
// the row stays in registers as raw 16-byte vectors (half the registers, more rows in flight) and
// is converted twice; otherwise the transformed fp32 values are kept.
// Plain rows (no rotation, no GELU), 16-bit input: warp per row in two streaming passes, amax
// then codes. The second pass re-reads the row from L2 (the rows in flight are a few MB), so
// registers stay few and many rows are in flight per SM.
template <typename T, bool SEG = false>
__global__ void __launch_bounds__(128, 12)
quant_rows_stream_kernel(const RowSrc src, int64_t M, int K, int8_t* __restrict__ q, float* __restrict__ s) {
  constexpr int kBatch = 4;
  const int lane = threadIdx.x & 31;
  const int nvec = K >> 3;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
       row += warps) {
    uint32_t am2 = 0u;
    for (int v0 = lane; v0 < nvec; v0 += 32 * kBatch) {
      uint4 raw[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int vi = v0 + 32 * b;
        raw[b] = vi < nvec ? __ldg(reinterpret_cast<const uint4*>(src_ptr<T, SEG>(src, row, vi * 8)))
                           : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        am2 = __vmaxu2(am2, __vmaxu2(__vmaxu2(raw[b].x & 0x7FFF7FFFu, raw[b].y & 0x7FFF7FFFu),
                                     __vmaxu2(raw[b].z & 0x7FFF7FFFu, raw[b].w & 0x7FFF7FFFu)));
      }
    }
    float amax = Vec8<T>::half_bits_to_float(max(am2 & 0xFFFFu, am2 >> 16));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = row_scale(amax, src.full_div);
    const float inv = __fdiv_rn(1.0f, scale);
    uint2* qr = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(K));
    for (int v0 = lane; v0 < nvec; v0 += 32 * kBatch) {
      uint4 raw[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int vi = v0 + 32 * b;
        raw[b] = vi < nvec ? __ldg(reinterpret_cast<const uint4*>(src_ptr<T, SEG>(src, row, vi * 8)))
                           : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int vi = v0 + 32 * b;
        if (vi < nvec) {
          float f[8];
          Vec8<T>::from_raw(raw[b], f);
          qr[vi] = quant8(f, scale, inv, src.full_div);
        }
      }
    }
    if (lane == 0) s[row] = scale;
  }
}

// Plain 16-bit rows (no rotation, no GELU), K <= 128 * 8 * VPT, K % 8 == 0, 16-byte aligned rows:
// one 128-thread CTA per row, each thread VPT 16-byte vectors held raw in registers (few registers,
// so 16 CTAs, the whole SM's 2048 threads, are resident and many rows' loads are in flight while
// other rows compute). The row's abs-max is a packed 16-bit max per thread, a warp reduction and a
// four-warp reduction through shared memory; then codes exactly as quant_rows_warp_kernel makes them.
template <typename T, int VPT, bool SEG = false>
__global__ void __launch_bounds__(128, 16)
quant_rows_cta_kernel(const RowSrc src, int64_t M, int K, int8_t* __restrict__ q, float* __restrict__ s) {
  __shared__ uint32_t red[2][4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nvec = K >> 3;
  int buf = 0;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x, buf ^= 1) {
    uint4 raw[VPT];
    uint32_t am2 = 0u;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = tid + 128 * i;
      raw[i] = vi < nvec ? *reinterpret_cast<const uint4*>(src_ptr<T, SEG>(src, row, vi * 8)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i)
      am2 = __vmaxu2(am2, __vmaxu2(__vmaxu2(raw[i].x & 0x7FFF7FFFu, raw[i].y & 0x7FFF7FFFu),
                                   __vmaxu2(raw[i].z & 0x7FFF7FFFu, raw[i].w & 0x7FFF7FFFu)));
    uint32_t hm = max(am2 & 0xFFFFu, am2 >> 16);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) hm = max(hm, __shfl_xor_sync(0xffffffffu, hm, o));
    if (lane == 0) red[buf][warp] = hm;
    __syncthreads();   // red[buf] is rewritten two rows later, after the next row's barrier
    hm = max(max(red[buf][0], red[buf][1]), max(red[buf][2], red[buf][3]));
    const float scale = row_scale(Vec8<T>::half_bits_to_float(hm), src.full_div);
    const float inv = __fdiv_rn(1.0f, scale);
    uint2* qr = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(K));
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = tid + 128 * i;
      if (vi < nvec) {
        float f[8];
        Vec8<T>::from_raw(raw[i], f);
        qr[vi] = quant8(f, scale, inv, src.full_div);
      }
    }
    if (tid == 0) s[row] = scale;
  }
}

template <typename T, int VPT, bool GROUP, int GELU, bool SEG = false>
__global__ void __launch_bounds__(128, 4)
quant_rows_warp_kernel(const RowSrc src, int64_t M, int K, int8_t* __restrict__ q, float* __restrict__ s) {
  constexpr bool kRaw = !GROUP && GELU == kGeluNone && sizeof(T) == 2;
  constexpr int kRawVecs = kRaw ? VPT : 1;
  constexpr int kFloatVecs = kRaw ? 1 : VPT;
  const int lane = threadIdx.x & 31;
  const int nvec = K >> 3;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
       row += warps) {
    uint4 raw[kRawVecs];
    float v[kFloatVecs][8];
    float am[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};   // independent max chains
    uint32_t am2[4] = {0u, 0u, 0u, 0u};                       // packed 16-bit |x| maxima (raw rows)
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + 32 * i;
      if (kRaw) {
        raw[kRaw ? i : 0] = vi < nvec ? *reinterpret_cast<const uint4*>(src_ptr<T, SEG>(src, row, vi * 8))
                                      : make_uint4(0, 0, 0, 0);
      } else {
        const int fi = kRaw ? 0 : i;
        if (vi < nvec) {
          Vec8<T>::load(src_ptr<T, SEG>(src, row, vi * 8), v[fi]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[fi][j] = 0.0f;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      if (kRaw) {
        // |x| of 16-bit floats: clear the sign bits; unsigned order then equals magnitude order,
        // so two lanes of a packed 16-bit max do two elements at a time.
        const uint4 u = raw[kRaw ? i : 0];
        am2[0] = __vmaxu2(am2[0], u.x & 0x7FFF7FFFu);
        am2[1] = __vmaxu2(am2[1], u.y & 0x7FFF7FFFu);
        am2[2] = __vmaxu2(am2[2], u.z & 0x7FFF7FFFu);
        am2[3] = __vmaxu2(am2[3], u.w & 0x7FFF7FFFu);
      } else {
        const int fi = kRaw ? 0 : i;
        if (GELU != kGeluNone) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[fi][j] = gelu_dtype<T>(v[fi][j], GELU);
        }
        // the 32 lanes at one i hold one 256-wide group (vectors 32 i .. 32 i + 31)
        if (GROUP) hadamard256_warp(v[fi], src.rot_order);
#pragma unroll
        for (int j = 0; j < 8; ++j) am[j] = fmaxf(am[j], fabsf(v[fi][j]));
      }
    }
    float amax = fmaxf(fmaxf(fmaxf(am[0], am[1]), fmaxf(am[2], am[3])), fmaxf(fmaxf(am[4], am[5]), fmaxf(am[6], am[7])));
    if (kRaw) {
      const uint32_t m2 = __vmaxu2(__vmaxu2(am2[0], am2[1]), __vmaxu2(am2[2], am2[3]));
      const uint32_t hmax = max(m2 & 0xFFFFu, m2 >> 16);
      amax = Vec8<T>::half_bits_to_float(hmax);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = row_scale(amax, src.full_div);
    const float inv = __fdiv_rn(1.0f, scale);
    int8_t* qr = q + row * static_cast<int64_t>(K);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) {
        uint2 w;
        if (kRaw) {
          float f[8];
          Vec8<T>::from_raw(raw[kRaw ? i : 0], f);
          w = quant8(f, scale, inv, src.full_div);
        } else {
          w = quant8(v[kRaw ? 0 : i], scale, inv, src.full_div);
        }
        *reinterpret_cast<uint2*>(qr + vi * 8) = w;
      }
    }
    if (lane == 0) s[row] = scale;
  }
}

constexpr int kQuantThreads = 128;

// Vector path: K % 8 == 0, ldx % 8 == 0 (elements), x 16-byte aligned. One CTA per row
// (grid-stride). Each thread holds up to VPT vectors of 8 elements. `group` is 0 or 256.
template <typename T, int VPT, bool GROUP, int GELU, bool SEG = false>
__global__ void __launch_bounds__(kQuantThreads)
quant_rows_kernel(const RowSrc src, int64_t M, int K, int8_t* __restrict__ q, float* __restrict__ s) {
  __shared__ float red[kQuantThreads / 32];
  const int tid = threadIdx.x;
  const int nvec = K >> 3;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    float v[VPT][8];
    float am4[4] = {0.0f, 0.0f, 0.0f, 0.0f};     // independent max chains
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = tid + i * kQuantThreads;
      if (vi < nvec) {
        Vec8<T>::load(src_ptr<T, SEG>(src, row, vi * 8), v[i]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
      }
      if (GELU != kGeluNone) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = gelu_dtype<T>(v[i][j], GELU);
      }
      // A 256-group is 32 consecutive vectors = the 32 lanes of one warp at one i. Groups
      // past the row end hold zeros and are discarded; every lane joins the shuffles.
      if (GROUP) hadamard256_warp(v[i], src.rot_order);
#pragma unroll
      for (int j = 0; j < 8; ++j) am4[j & 3] = fmaxf(am4[j & 3], fabsf(v[i][j]));
    }
    float amax = fmaxf(fmaxf(am4[0], am4[1]), fmaxf(am4[2], am4[3]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((tid & 31) == 0) red[tid >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < kQuantThreads / 32; ++w) amax = fmaxf(amax, red[w]);
    __syncthreads();
    const float scale = row_scale(amax, src.full_div);
    const float inv = __fdiv_rn(1.0f, scale);
    int8_t* qr = q + row * static_cast<int64_t>(K);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = tid + i * kQuantThreads;
      if (vi < nvec) *reinterpret_cast<uint2*>(qr + vi * 8) = quant8(v[i], scale, inv, src.full_div);
    }
    if (tid == 0) s[row] = scale;
  }
}

// Generic path for any K and stride (no rotation): two passes over the row.
template <typename T, int GELU>
__global__ void __launch_bounds__(kQuantThreads)
quant_rows_scalar_kernel(const T* __restrict__ x, int64_t M, int K, int64_t ldx, int8_t* __restrict__ q,
                         float* __restrict__ s, int full_div) {
  __shared__ float red[kQuantThreads / 32];
  const int tid = threadIdx.x;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const T* xr = x + row * ldx;
    float amax = 0.0f;
    for (int c = tid; c < K; c += kQuantThreads) {
      float t = Vec8<T>::one(xr + c);
      if (GELU != kGeluNone) t = gelu_dtype<T>(t, GELU);
      amax = fmaxf(amax, fabsf(t));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((tid & 31) == 0) red[tid >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < kQuantThreads / 32; ++w) amax = fmaxf(amax, red[w]);
    __syncthreads();
    const float scale = row_scale(amax, full_div);
    int8_t* qr = q + row * static_cast<int64_t>(K);
    for (int c = tid; c < K; c += kQuantThreads) {
      float t = Vec8<T>::one(xr + c);
      if (GELU != kGeluNone) t = gelu_dtype<T>(t, GELU);
      qr[c] = quant_code(t, scale, full_div);
    }
    if (tid == 0) s[row] = scale;
  }
}

}  // namespace dc
